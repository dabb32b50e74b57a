"""Matrix sharding of the optimizer step across the ranks of a process group.

One process per GPU.  Every rank holds the whole model and runs the hooks on
its own microbatches; at step():
  1. reduce_statistics: the accumulated statistic sums and row counts of all
     selected matrices are summed over the group with one flat all-reduce, so
     every rank finishes identical whiteners (as one large batch would);
  2. each rank runs momentum -> whitening -> S8 -> mapback -> update only for
     the matrices it owns (partition "lpt": longest-processing-time greedy
     over S8 FLOPs; "layer": contiguous transformer layers per rank);
  3. exchange: the owners' updated FP32 weights are all-gathered with one
     padded all_gather_into_tensor and copied back into every rank's params.
There is no other data-path collective; gradients are averaged by the
caller's data-parallel wrapper as usual.
"""
from __future__ import annotations

import re

import torch
import torch.distributed as dist

from .workloads import s8_executed_flops

_LAYER = re.compile(r"\.h\.(\d+)\.")


def partition_matrices(named_shapes: dict[str, tuple[int, int]], world: int, how: str = "lpt") -> dict[str, int]:
    """Owner rank of each matrix name."""
    names = list(named_shapes)
    if world <= 1:
        return {n: 0 for n in names}
    if how == "layer":
        layers = {}
        for n in names:
            m = _LAYER.search(n)
            layers[n] = int(m.group(1)) if m else -1
        distinct = sorted(set(layers.values()))
        index = {layer: i for i, layer in enumerate(distinct)}
        return {n: index[layers[n]] * world // len(distinct) for n in names}
    if how != "lpt":
        raise ValueError(f"unknown partition {how!r} (expected 'lpt' or 'layer')")
    cost = {n: s8_executed_flops([named_shapes[n]]) for n in names}
    load = [0.0] * world
    owner = {}
    for n in sorted(names, key=lambda k: (-cost[k], names.index(k))):
        r = min(range(world), key=lambda i: (load[i], i))
        owner[n] = r
        load[r] += cost[n]
    return owner


class MatrixSharding:
    def __init__(self, opt, group, *, partition: str = "lpt"):
        self.opt = opt
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        shapes = {n: tuple(p.shape) for n, p in opt.named_matrices.items()}
        self.owner_by_name = partition_matrices(shapes, self.world, partition)
        self._owner = {id(opt.named_matrices[n]): r for n, r in self.owner_by_name.items()}
        self._gather = None

    def owns(self, parameter) -> bool:
        return self._owner[id(parameter)] == self.rank

    def owner(self, parameter) -> int:
        return self._owner[id(parameter)]

    # ------------------------------------------------------ statistics
    def reduce_statistics(self, matrix_items) -> None:
        """Sums statistic vectors and row counts over the group."""
        if self.world == 1 or not matrix_items:
            return
        opt = self.opt
        seen, tensors, counters = set(), [], []
        for parameter, source, _ in matrix_items:
            if id(source) not in seen:
                seen.add(id(source))
                st = opt.state[source]
                tensors.append(st["a_sum"])
                if opt.rank_one_a:
                    tensors.append(st["a_first_sum"])
                counters.append((st, "a_count"))
            st = opt.state[parameter]
            tensors.append(st["b_sum"])
            counters.append((st, "b_count"))
        flat = torch.cat([t.reshape(-1) for t in tensors])
        counts = torch.tensor([st[key] for st, key in counters], dtype=torch.float64, device=flat.device)
        dist.all_reduce(flat, group=self.group)
        dist.all_reduce(counts, group=self.group)
        offset = 0
        for t in tensors:
            t.copy_(flat[offset:offset + t.numel()].view_as(t))
            offset += t.numel()
        for (st, key), value in zip(counters, counts.tolist()):
            st[key] = int(round(value))

    # --------------------------------------------------------- weights
    def exchange(self, matrix_items) -> None:
        """All-gathers every matrix from its owner into all ranks."""
        if self.world == 1 or not matrix_items:
            return
        params = [item[0] for item in matrix_items]
        key = tuple(id(p) for p in params)
        if self._gather is None or self._gather[0] != key:
            per_rank = [[] for _ in range(self.world)]
            for p in params:
                per_rank[self.owner(p)].append(p)
            shard = max(sum(p.numel() for p in ps) for ps in per_rank)
            device = params[0].device
            send = torch.empty(shard, dtype=torch.float32, device=device)
            recv = torch.empty(shard * self.world, dtype=torch.float32, device=device)
            self._gather = (key, per_rank, send, recv, shard)
        _, per_rank, send, recv, shard = self._gather
        offset = 0
        for p in per_rank[self.rank]:
            send[offset:offset + p.numel()].copy_(p.detach().reshape(-1))
            offset += p.numel()
        dist.all_gather_into_tensor(recv, send, group=self.group)
        with torch.no_grad():
            for r, ps in enumerate(per_rank):
                if r == self.rank:
                    continue
                offset = r * shard
                for p in ps:
                    p.copy_(recv[offset:offset + p.numel()].view_as(p))
                    offset += p.numel()
