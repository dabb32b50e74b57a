"""Matrix sharding of the optimizer step across the ranks of a process group.

One process per GPU.  Every rank holds the whole model and runs the hooks on
its own microbatches; at step():
  1. reduce_statistics: the accumulated statistic sums and row counts of all
     selected matrices are summed over the group (one flat all-reduce plus a
     small one for the counts, which stay on the device), so every rank
     finishes identical whiteners (as one large batch would);
  2. each rank runs momentum -> whitening -> S8 -> mapback -> update only for
     the matrices it owns (partition "lpt": longest-processing-time greedy
     over S8 FLOPs; "layer": contiguous transformer layers per rank);
  3. exchange: the owners' updated FP32 weights are all-gathered with one
     padded all_gather_into_tensor and copied back into every rank's params
     (exchange="weights", the default).  exchange="bf16_delta" gathers the
     update deltas lr * direction rounded to BF16 instead (half the NVLink
     bytes); every rank, the owner included, subtracts the same rounded delta,
     so the ranks stay bitwise identical.  The rounding (2^-9 relative per
     element) perturbs the update direction far inside its 1e-2 tolerance.
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


EXCHANGES = ("weights", "bf16_delta")


class MatrixSharding:
    def __init__(self, opt, group, *, partition: str = "lpt", exchange: str = "weights"):
        if exchange not in EXCHANGES:
            raise ValueError(f"unknown exchange {exchange!r} (expected one of {EXCHANGES})")
        self.opt = opt
        self.group = group
        self.exchange_mode = exchange
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
    def reduce_statistics(self, tensors: list[torch.Tensor], counts: list[int]) -> torch.Tensor | None:
        """Sums the statistic vectors (in place) and their row counts over the
        group; returns the summed counts as an int64 tensor on the tensors'
        device, read by the statistics kernel without a host synchronisation.
        None for a single rank."""
        if self.world == 1 or not tensors:
            return None
        total = torch.tensor(counts, dtype=torch.int64).to(tensors[0].device, non_blocking=True)
        if len(tensors) == 1:
            dist.all_reduce(tensors[0], group=self.group)  # the optimizer's flat statistic buffer
        else:
            flat = torch.cat([t.reshape(-1) for t in tensors])
            dist.all_reduce(flat, group=self.group)
            offset = 0
            for t in tensors:
                t.copy_(flat[offset:offset + t.numel()].view_as(t))
                offset += t.numel()
        dist.all_reduce(total, group=self.group)
        return total

    # --------------------------------------------------------- weights
    def _layout(self):
        """Static all-gather layout: each rank's owned matrices back to back in
        its send slot of `shard` floats (every selected matrix, every step)."""
        if self._gather is None:
            params = list(self.opt.named_matrices.values())
            per_rank = [[] for _ in range(self.world)]
            for p in params:
                per_rank[self.owner(p)].append(p)
            # 4-element alignment keeps every slot 16-byte (FP32) / 8-byte (BF16) aligned
            shard = max(sum((p.numel() + 3) // 4 * 4 for p in ps) for ps in per_rank)
            device = params[0].device
            dtype = torch.bfloat16 if self.exchange_mode == "bf16_delta" else torch.float32
            send = torch.zeros(shard, dtype=dtype, device=device)
            recv = torch.empty(shard * self.world, dtype=dtype, device=device)
            slots, unpack = {}, []
            for r, ps in enumerate(per_rank):
                offset = 0
                for p in ps:
                    if r == self.rank:
                        slots[id(p)] = send[offset:offset + p.numel()].view_as(p)
                    else:
                        unpack.append((p, recv[r * shard + offset:r * shard + offset + p.numel()]))
                    offset += (p.numel() + 3) // 4 * 4
            self._gather = (send, recv, slots, unpack)
        return self._gather

    @property
    def export_mode(self) -> int:
        """The plan's export mode for this exchange (see StepPlan)."""
        from . import _lib
        return _lib.SM_EXPORT_BF16_DELTA if self.exchange_mode == "bf16_delta" else _lib.SM_EXPORT_WEIGHTS

    def send_slot(self, parameter) -> torch.Tensor | None:
        """Where the step also writes an owned matrix's updated weight, or its
        BF16 update delta (its all-gather send slot); None for a single rank."""
        if self.world == 1:
            return None
        return self._layout()[2][id(parameter)]

    def exchange(self, matrix_items) -> None:
        """All-gathers every matrix from its owner into all ranks.  The owners'
        send slots were filled by the update kernel itself; the received
        weights are scattered back with one multi-tensor copy launch, or the
        received BF16 deltas of the matrices stepped now are subtracted with
        one multi-tensor launch."""
        if self.world == 1:
            return
        from .engine import apply_bf16_delta_multi, copy_multi
        send, recv, slots, unpack = self._layout()
        dist.all_gather_into_tensor(recv, send, group=self.group)
        if self.exchange_mode == "bf16_delta":
            # only the matrices stepped now: a skipped matrix's slot holds an old delta
            stepped = {id(item[0]) for item in matrix_items}
            apply_bf16_delta_multi([(p.detach(), src) for p, src in unpack if id(p) in stepped], recv.device)
        else:
            copy_multi([(p.detach(), src) for p, src in unpack], recv.device)
