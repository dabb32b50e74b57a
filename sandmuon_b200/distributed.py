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
  3. exchange: every rank keeps the selected matrices in one flat FP32
     buffer of the same layout (each owner's matrices back to back in its
     shard).  With exchange="weights" (the default) the owners' updated
     weights reach the other ranks one of two ways (`transport`):
       "peer": the update kernel itself stores each updated weight into
       every rank's copy of the buffer (CUDA IPC mappings of the peers'
       buffers, plain stores over NVLink), and the exchange is a one-element
       all-reduce that orders the ranks: no bulk collective at all;
       "nccl": an in-place all_gather_into_tensor of the buffer.
     "auto" (the default) takes "peer" when the buffer is on CUDA under an
     NCCL group and every rank could map every peer, else "nccl".
     exchange="bf16_delta" gathers the
     update deltas lr * direction rounded to BF16 instead (half the NVLink
     bytes); every rank, the owner included, subtracts the same rounded delta,
     so the ranks stay bitwise identical.  The rounding (2^-9 relative per
     element) perturbs the update direction far inside its 1e-2 tolerance.
Gradients are averaged by the caller's data-parallel wrapper as usual, or,
with reduce_gradients=True on the optimizer, by reduce_gradients below:
every matrix gradient is reduce-scattered to its owner (half the bytes of an
all-reduce; only the owner steps that matrix) and the auxiliary gradients are
all-reduced.  Momentum buffers exist only on a matrix's owner (ZeRO-1 style);
consolidated_momentum gathers them for a checkpoint in the reference layout.
"""
from __future__ import annotations

import re

import torch
import torch.distributed as dist

from .workloads import s8_dense_flops

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
    cost = {n: s8_dense_flops([named_shapes[n]]) for n in names}
    load = [0.0] * world
    owner = {}
    for n in sorted(names, key=lambda k: (-cost[k], names.index(k))):
        r = min(range(world), key=lambda i: (load[i], i))
        owner[n] = r
        load[r] += cost[n]
    return owner


EXCHANGES = ("weights", "bf16_delta")
TRANSPORTS = ("auto", "peer", "nccl")


def _copy_pairs(pairs, device) -> None:
    """dst.copy_(src) for same-size CUDA tensors, one library launch per 64."""
    from .engine import copy_multi
    copy_multi(pairs, device)


class MatrixSharding:
    """copy_fn(pairs, device) performs the packing copies (dst, src) of the
    gradient reduction and the momentum gather; the default is the library's
    multi-tensor copy kernel.  With exchange="weights" (and more than one
    rank) the constructor moves the selected matrices' storage into the flat
    all-gather buffer (_rehome_weights)."""

    def __init__(self, opt, group, *, partition: str = "lpt", exchange: str = "weights", copy_fn=None,
                 transport: str = "auto"):
        if exchange not in EXCHANGES:
            raise ValueError(f"unknown exchange {exchange!r} (expected one of {EXCHANGES})")
        if transport not in TRANSPORTS:
            raise ValueError(f"unknown transport {transport!r} (expected one of {TRANSPORTS})")
        self.opt = opt
        self.group = group
        self.exchange_mode = exchange
        self._copy = copy_fn or _copy_pairs
        self._grad_bufs = None
        self._aux_bufs = {}
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        shapes = {n: tuple(p.shape) for n, p in opt.named_matrices.items()}
        self.owner_by_name = partition_matrices(shapes, self.world, partition)
        self._owner = {id(opt.named_matrices[n]): r for n, r in self.owner_by_name.items()}
        self._gather = None
        self._flat_weights = None
        self.peer_bases: list[int] = []   # the other ranks' flat buffers, mapped here
        self._opened: list[int] = []      # IPC bases to unmap at close
        self._token = None
        if exchange == "weights" and self.world > 1:
            self._rehome_weights()
            if transport != "nccl":
                self._map_peers(required=transport == "peer")

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

    # ------------------------------------------------------- gradients
    def _slots(self):
        """(shard, {id(p): (owner, offset)}): every matrix at a 4-element
        aligned offset inside its owner's segment of `shard` elements."""
        if not hasattr(self, "_slot_map"):
            offsets, fill = {}, [0] * self.world
            for p in self.opt.named_matrices.values():
                r = self.owner(p)
                offsets[id(p)] = (r, fill[r])
                fill[r] += (p.numel() + 3) // 4 * 4
            self._slot_map = (max(fill), offsets)
        return self._slot_map

    def _average_op(self):
        """(averages?, op) for an averaging collective: NCCL averages inside
        the collective; other backends sum, and the caller divides."""
        avg = dist.get_backend(self.group) == "nccl"
        return avg, (dist.ReduceOp.AVG if avg else dist.ReduceOp.SUM)

    def reduce_gradients(self, matrix_items, aux_params) -> dict:
        """Averages gradients over the group.  Matrix gradients are packed by
        owner and reduce-scattered, so each rank receives the average of the
        matrices it owns (returned as {id(p): averaged gradient view}; the
        other ranks' .grad of those matrices stay local).  Auxiliary
        gradients are all-reduced in place."""
        if self.world == 1:
            return {}
        shard, offsets = self._slots()
        params = [item[0] for item in matrix_items]
        device = params[0].device if params else (aux_params[0].device if aux_params else None)
        out = {}
        if params:
            if self._grad_bufs is None or self._grad_bufs[0].device != device:
                self._grad_bufs = (torch.empty(shard * self.world, dtype=torch.float32, device=device),
                                   torch.empty(shard, dtype=torch.float32, device=device))
            send, recv = self._grad_bufs
            pairs = []
            for p in params:
                r, off = offsets[id(p)]
                pairs.append((send[r * shard + off:r * shard + off + p.numel()], p.grad.reshape(-1)))
                if r == self.rank:
                    out[id(p)] = recv[off:off + p.numel()].view_as(p)
            self._copy(pairs, device)
            avg, op = self._average_op()
            dist.reduce_scatter_tensor(recv, send, op=op, group=self.group)
            if not avg:
                recv.div_(self.world)
        if aux_params:
            total = sum(p.numel() for p in aux_params)
            buf = self._aux_bufs.get(device)
            if buf is None or buf.numel() < total:
                buf = torch.empty(total, dtype=torch.float32, device=device)
                self._aux_bufs[device] = buf
            views, off = [], 0
            for p in aux_params:
                views.append((buf[off:off + p.numel()], p.grad.reshape(-1)))
                off += p.numel()
            self._copy(views, device)
            flat = buf[:total]
            avg, op = self._average_op()
            dist.all_reduce(flat, op=op, group=self.group)
            if not avg:
                flat.div_(self.world)
            self._copy([(g, v) for v, g in views], device)
        return out

    def consolidated_momentum(self) -> dict:
        """{id(p): momentum_buffer} of every selected matrix that has one on
        its owner, all-gathered so every rank holds all of them (the
        reference's state layout, for a checkpoint)."""
        shard, offsets = self._slots()
        params = list(self.opt.named_matrices.values())
        have = torch.tensor([1 if (self.owns(p) and "momentum_buffer" in self.opt.state.get(p, {})) else 0
                             for p in params], dtype=torch.int32)
        device = params[0].device
        if dist.get_backend(self.group) == "nccl":
            have = have.to(device)
        dist.all_reduce(have, group=self.group)
        have = have.cpu().tolist()
        send = torch.zeros(shard, dtype=torch.float32, device=device)
        recv = torch.empty(shard * self.world, dtype=torch.float32, device=device)
        pairs = []
        for p, h in zip(params, have):
            r, off = offsets[id(p)]
            if h and r == self.rank:
                pairs.append((send[off:off + p.numel()], self.opt.state[p]["momentum_buffer"].reshape(-1)))
        if pairs:
            self._copy(pairs, device)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        out = {}
        for p, h in zip(params, have):
            if h:
                r, off = offsets[id(p)]
                out[id(p)] = recv[r * shard + off:r * shard + off + p.numel()].view_as(p).clone()
        return out

    # --------------------------------------------------------- weights
    def _rehome_weights(self):
        """exchange="weights": every selected matrix becomes a view of one flat
        FP32 buffer laid out as the all-gather's output (each owner's matrices
        back to back in its shard, shards padded to the largest), so the
        update kernel writes owned weights straight into the gathered layout
        and the all-gather runs in place: no export copy of the owned weights
        and no scatter of the received ones.  The parameters keep their
        identity (only their storage moves); they must be contiguous float32.
        A matrix not stepped this time travels as its current value."""
        shard, offsets = self._slots()
        params = list(self.opt.named_matrices.values())
        for p in params:
            if p.dtype != torch.float32 or not p.is_contiguous():
                raise TypeError("a sharded sandmuon_b200 optimizer needs contiguous float32 matrix parameters; "
                                f"got {p.dtype} {'contiguous' if p.is_contiguous() else 'strided'}")
        flat = torch.zeros(shard * self.world, dtype=torch.float32, device=params[0].device)
        with torch.no_grad():
            for p in params:
                r, off = offsets[id(p)]
                view = flat[r * shard + off:r * shard + off + p.numel()].view_as(p)
                view.copy_(p)
                p.data = view
        self._flat_weights = flat
        self._homes = [(p, p.data_ptr()) for p in params]

    def _map_peers(self, required: bool) -> None:
        """Maps every other rank's flat weight buffer into this device (CUDA
        IPC; a collective).  All ranks agree: if any rank cannot map every
        peer, every rank unmaps and keeps the NCCL all-gather (or raises when
        `required`)."""
        from . import _lib
        flat = self._flat_weights
        device = flat.device
        usable = flat.is_cuda and dist.get_backend(self.group) == "nccl" and self.world - 1 <= 15
        entry = None
        if usable:
            try:
                entry = _lib.ipc_export(flat)
            except RuntimeError:
                entry = None
        entries = [None] * self.world
        dist.all_gather_object(entries, entry, group=self.group)
        ok = all(e is not None for e in entries)
        bases = []
        if ok:
            try:
                for r, (handle, offset) in enumerate(entries):
                    if r == self.rank:
                        continue
                    base = _lib.ipc_open(handle, device)
                    self._opened.append(base)
                    bases.append(base + offset)
            except RuntimeError:
                ok = False
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device if flat.is_cuda else "cpu")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        if int(flag.item()) != 1:
            self._unmap()
            if required:
                raise RuntimeError("transport='peer' needs every rank to map every peer's weight buffer "
                                   "(CUDA tensors, an NCCL group, at most 16 ranks)")
            return
        self.peer_bases = bases
        self._token = torch.zeros(1, dtype=torch.float32, device=device)

    def _unmap(self) -> None:
        from . import _lib
        for base in self._opened:
            _lib.ipc_close(base, self._flat_weights.device)
        self._opened = []
        self.peer_bases = []

    def peer_target(self) -> tuple[int, int, list[int]]:
        """(local flat buffer address, its bytes, the peers' buffer addresses)
        for StepPlan.set_peers."""
        flat = self._flat_weights
        return flat.data_ptr(), flat.numel() * flat.element_size(), list(self.peer_bases)

    def close(self) -> None:
        """Unmaps the peers' buffers after a barrier, so that no rank still
        stores into a buffer another rank is about to free (a collective)."""
        if self._opened:
            dist.all_reduce(self._token, group=self.group)
            torch.cuda.synchronize(self._flat_weights.device)
            self._unmap()

    def _layout(self):
        """(send, recv, slots, unpack) of the all-gather.  Weights: send is this
        rank's shard of the flat weight buffer and recv the whole buffer (an
        in-place all-gather); slots are the owned parameters themselves and
        nothing is unpacked.  BF16 deltas: each rank's owned matrices' deltas
        back to back in its send slot of `shard` elements; unpack pairs every
        other matrix with its gathered delta."""
        if self._gather is None:
            shard, offsets = self._slots()
            params = list(self.opt.named_matrices.values())
            if self.exchange_mode == "weights":
                flat = self._flat_weights
                send = flat[self.rank * shard:(self.rank + 1) * shard]
                slots = {id(p): p.detach() for p in params if self.owns(p)}
                self._gather = (send, flat, slots, [])
            else:
                device = params[0].device
                send = torch.zeros(shard, dtype=torch.bfloat16, device=device)
                recv = torch.empty(shard * self.world, dtype=torch.bfloat16, device=device)
                slots, unpack = {}, []
                for p in params:
                    r, off = offsets[id(p)]
                    if r == self.rank:
                        slots[id(p)] = send[off:off + p.numel()].view_as(p)
                    else:
                        unpack.append((p, recv[r * shard + off:r * shard + off + p.numel()]))
                self._gather = (send, recv, slots, unpack)
        return self._gather

    @property
    def export_mode(self) -> int:
        """The plan's export mode for this exchange (see StepPlan)."""
        from . import _lib
        return _lib.SM_EXPORT_BF16_DELTA if self.exchange_mode == "bf16_delta" else _lib.SM_EXPORT_WEIGHTS

    def send_slot(self, parameter) -> torch.Tensor | None:
        """Where the step also writes an owned matrix's BF16 update delta (its
        all-gather send slot); None for the weight exchange (the weights are
        gathered in place) and for a single rank."""
        if self.world == 1 or self.exchange_mode == "weights":
            return None
        return self._layout()[2][id(parameter)]

    def exchange(self, matrix_items) -> None:
        """Brings the owners' updates to all ranks.  Weights by peer stores:
        a one-element all-reduce that orders the ranks.  Weights by NCCL: one
        in-place all-gather of the flat weight buffer (the update kernel
        already wrote the owned weights there).  BF16 deltas: the owners' send
        slots were filled by the update kernel; the received deltas of the
        matrices stepped now are subtracted with one multi-tensor launch (a
        slot of a matrix its owner did not step holds an older delta).  The
        all-gather runs on every rank whenever step() runs, whatever was
        stepped, so the ranks' collectives stay paired."""
        if self.world == 1:
            return
        from .engine import apply_bf16_delta_multi
        if self.exchange_mode == "weights":
            for p, ptr in self._homes:
                if p.data_ptr() != ptr:
                    raise RuntimeError("a selected matrix's storage moved after the sharded optimizer was built "
                                       "(for example model.to() or a reassigned .data); build the optimizer "
                                       "after the model is in place")
        if self.peer_bases:
            # the update kernel already stored every owner's weights into every
            # rank's buffer: this all-reduce only orders the ranks (each rank's
            # update kernel precedes its part of it in stream order)
            dist.all_reduce(self._token, group=self.group)
            return
        send, recv, slots, unpack = self._layout()
        dist.all_gather_into_tensor(recv, send, group=self.group)
        if self.exchange_mode == "bf16_delta":
            stepped = {id(item[0]) for item in matrix_items}
            apply_bf16_delta_multi([(p.detach(), src) for p, src in unpack if id(p) in stepped], recv.device)
