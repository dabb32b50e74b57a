"""Worker for tests/test_gpu_multi.py: one rank of a sharded optimizer step.

Launched by torch.distributed.run (one process per GPU) with the output
directory, the partition ("lpt" / "layer"), the exchange ("weights" /
"bf16_delta") and optionally "reduce".  Every rank builds the same mini
GPT-named model, injects the same statistics and gradients (with "reduce":
rank-dependent gradients averaging to them, which the optimizer reduces
itself), runs two sharded steps (statistic all-reduce, owned-matrix S8,
exchange) and saves its weights and consolidated momentum buffers to
<out_dir>/rank<r>.pt (rank 0 also the initial weights to init.pt).
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


def main(out_dir: str, partition: str, exchange: str, reduce: bool):
    from sandmuon_b200 import RankOneAWeightedPE
    from sandmuon_b200.workloads import gpt_matrix_model, synth_gpt_statistics
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        torch.manual_seed(5)
        model = gpt_matrix_model(3, 256, 1024).to(device)
        if rank == 0:
            torch.save({n: p.detach().cpu() for n, p in model.named_parameters()}, Path(out_dir) / "init.pt")
        opt = RankOneAWeightedPE(model, lr=1e-2, process_group=dist.group.WORLD, partition=partition,
                                 exchange=exchange, reduce_gradients=reduce)
        rng = np.random.default_rng(5)
        world = dist.get_world_size()
        for step in range(2):
            synth_gpt_statistics(opt, rng, count=4096)
            for p in model.parameters():
                g = (rng.standard_normal(tuple(p.shape)) * 1e-4).astype(np.float32)
                if reduce:  # rank-dependent gradients whose average over the ranks is g
                    g = g * np.float32(2.0 * (rank + 1) / (world + 1))
                p.grad = torch.from_numpy(g).to(device)
            opt.step()
        torch.cuda.synchronize()
        out = {n: p.detach().cpu() for n, p in model.named_parameters()}
        state = opt.consolidated_state_dict()
        names = [n for n, _ in model.named_parameters()]
        for i, st in state["state"].items():
            if "momentum_buffer" in st:
                out[names[i] + "/momentum"] = st["momentum_buffer"].detach().cpu()
        torch.save(out, Path(out_dir) / f"rank{rank}.pt")
        opt.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "lpt", sys.argv[3] if len(sys.argv) > 3 else "weights",
         len(sys.argv) > 4 and sys.argv[4] == "reduce")
