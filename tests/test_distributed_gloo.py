"""Multi-rank host logic of the matrix sharding on CPU with gloo, world size 2.

The CUDA step is replaced by a test-only stub (a deterministic per-owner
update), so these tests check partitioning, the statistic all-reduce and the
weight exchange without a GPU.  The stub exists only here, not in the product.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sandmuon_b200.distributed import MatrixSharding, partition_matrices
from sandmuon_b200.workloads import gpt_matrix_model, s8_dense_flops


def test_unknown_exchange_is_rejected():
    with pytest.raises(ValueError):
        MatrixSharding(None, None, exchange="fp8")


def test_lpt_partition_balances_s8_flops():
    shapes = {f"transformer.h.{l}.attn.{p}.weight": (768, 768) for l in range(9)
              for p in ("q_proj", "k_proj", "v_proj", "o_proj")}
    shapes.update({f"transformer.h.{l}.mlp.c_fc.weight": (3072, 768) for l in range(9)})
    shapes.update({f"transformer.h.{l}.mlp.c_proj.weight": (768, 3072) for l in range(9)})
    for world in (1, 2, 4, 8):
        owner = partition_matrices(shapes, world, "lpt")
        load = [0.0] * world
        for n, r in owner.items():
            load[r] += s8_dense_flops([shapes[n]])
        assert set(owner) == set(shapes) and set(owner.values()) <= set(range(world))
        assert max(load) / (sum(load) / world) < 1.2
        by_layer = partition_matrices(shapes, world, "layer")
        layers = {}
        for n, r in by_layer.items():
            layers.setdefault(n.split(".")[2], set()).add(r)
        assert all(len(rs) == 1 for rs in layers.values())
    with pytest.raises(ValueError):
        partition_matrices(shapes, 2, "round_robin")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _StubOptimizer:
    """The attributes MatrixSharding reads from an optimizer."""

    def __init__(self, model):
        from sandmuon_b200.optimizer import _QKV_SHARING
        self.named_matrices = {n + ".weight": m.weight for n, m in model.named_modules()
                               if isinstance(m, torch.nn.Linear)}
        self.rank_one_a = True
        self.state = {}
        self.a_sources = {id(p): p for p in self.named_matrices.values()}
        for name, p in self.named_matrices.items():
            match = _QKV_SHARING.match(name)
            if match:
                self.a_sources[id(p)] = self.named_matrices[match.group(1) + "q_proj.weight"]


def _worker(rank, world, port, partition, results, exchange="weights"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = gpt_matrix_model(3, 16, 64)
        opt = _StubOptimizer(model)
        sharding = MatrixSharding(opt, dist.group.WORLD, partition=partition, exchange=exchange)
        items = []
        for name, p in opt.named_matrices.items():
            src = opt.a_sources[id(p)]
            st_src = opt.state.setdefault(src, {})
            if "a_sum" not in st_src:
                st_src.update(a_sum=torch.full((p.shape[1],), float(rank + 1)),
                              a_first_sum=torch.full((p.shape[1],), float(rank)), a_count=10 * (rank + 1))
            st = opt.state.setdefault(p, {})
            st.update(b_sum=torch.full((p.shape[0],), 2.0 * (rank + 1)), b_count=10 * (rank + 1))
            items.append((p, src, {}))
        seen, tensors, counters = set(), [], []
        for p, src, _ in items:
            if id(src) not in seen:
                seen.add(id(src))
                tensors += [opt.state[src]["a_sum"], opt.state[src]["a_first_sum"]]
                counters.append((opt.state[src], "a_count"))
            tensors.append(opt.state[p]["b_sum"])
            counters.append((opt.state[p], "b_count"))
        total = sharding.reduce_statistics(tensors, [st[k] for st, k in counters])
        for (st, k), v in zip(counters, total.tolist()):
            st[k] = v
        send, recv, slots, unpack = sharding._layout()
        if exchange == "weights":
            # test-only compute stub: each owner writes a value unique to (matrix, owner)
            with torch.no_grad():
                for i, (p, _, _) in enumerate(items):
                    p.fill_(100.0 * i + sharding.rank if sharding.owns(p) else -1.0)
            # the matrices live in the flat gather buffer: an owned slot is the
            # parameter itself, and the in-place all-gather delivers the rest
            assert not unpack and recv.data_ptr() <= send.data_ptr() < recv.data_ptr() + recv.numel() * 4
            for p, _, _ in items:
                if sharding.owns(p):
                    assert sharding.send_slot(p) is None
                    assert slots[id(p)].data_ptr() == p.data_ptr()
            dist.all_gather_into_tensor(recv, send, group=dist.group.WORLD)
        else:
            # every rank starts from the same weights; each owner subtracts its
            # BF16 delta (a value unique to matrix and owner) and exports it;
            # the others subtract the gathered delta, as exchange() does
            assert send.dtype == torch.bfloat16
            with torch.no_grad():
                for i, (p, _, _) in enumerate(items):
                    p.fill_(1000.0)
                    if sharding.owns(p):
                        delta = torch.full_like(p, 2.0 * i + sharding.rank).to(torch.bfloat16)  # exact in BF16
                        slots[id(p)].copy_(delta)
                        p.sub_(delta.float())
            dist.all_gather_into_tensor(recv, send, group=dist.group.WORLD)
            with torch.no_grad():
                for p, src in unpack:
                    p.sub_(src.view_as(p).float())
                for i, (p, _, _) in enumerate(items):
                    p.copy_(1000.0 - p)  # back to the delta value for the shared assertions
        out = {}
        for i, (p, src, _) in enumerate(items):
            out[i] = (float(p.min()), float(p.max()), sharding.owner(p),
                      float(opt.state[src]["a_sum"][0]), float(opt.state[src]["a_first_sum"][0]),
                      opt.state[src]["a_count"], float(opt.state[p]["b_sum"][0]), opt.state[p]["b_count"])
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("partition,exchange", [("lpt", "weights"), ("layer", "weights"), ("lpt", "bf16_delta")])
def test_two_rank_statistics_reduction_and_weight_exchange(partition, exchange):
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, partition, results, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    r0, r1 = results[0], results[1]
    assert r0 == r1                       # every rank ends with identical weights and statistics
    owners = {v[2] for v in r0.values()}
    assert owners == {0, 1}
    for i, (lo, hi, owner, a_sum, a_first, a_count, b_sum, b_count) in r0.items():
        expected = 100.0 * i + owner if exchange == "weights" else 2.0 * i + owner
        assert lo == hi == expected  # the owner's update reached every rank
        assert a_sum == 1.0 + 2.0 and a_first == 0.0 + 1.0 and a_count == 30
        assert b_sum == 2.0 + 4.0 and b_count == 30


def _torch_copy(pairs, device):
    """Test-only stand-in for the library's multi-tensor copy kernel."""
    for dst, src in pairs:
        dst.copy_(src.reshape(dst.shape))


def _grad_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = gpt_matrix_model(3, 16, 64)
        opt = _StubOptimizer(model)
        sharding = MatrixSharding(opt, dist.group.WORLD, partition="lpt", copy_fn=_torch_copy)
        params = list(opt.named_matrices.values())
        aux = [torch.nn.Parameter(torch.zeros(5, 3)), torch.nn.Parameter(torch.zeros(7))]
        for i, p in enumerate(params):
            p.grad = torch.full_like(p, float(i + 1) * (rank + 1))     # rank-dependent gradients
        for i, p in enumerate(aux):
            p.grad = torch.full_like(p, 10.0 * (i + 1) * (rank + 1))
        index = {id(p): i for i, p in enumerate(params)}
        averaged = sharding.reduce_gradients([(p, p, {}) for p in params], aux)
        out = {"owned": sorted(index[k] for k in averaged),
               "avg": {index[k]: (float(v.min()), float(v.max())) for k, v in averaged.items()},
               "aux": [(float(p.grad.min()), float(p.grad.max())) for p in aux]}
        # momentum only on owners; the consolidated gather gives every rank all of them
        for i, p in enumerate(params):
            if sharding.owns(p):
                opt.state.setdefault(p, {})["momentum_buffer"] = torch.full_like(p, 0.5 * i)
        moms = sharding.consolidated_momentum()
        out["moms"] = {index[k]: (float(v.min()), float(v.max())) for k, v in moms.items()}
        out["owners"] = [sharding.owner(p) for p in params]
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_two_rank_gradient_reduce_scatter_and_momentum_gather():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    r0, r1 = results[0], results[1]
    owners = r0["owners"]
    assert owners == r1["owners"] and set(owners) == {0, 1}
    for rank, res in ((0, r0), (1, r1)):
        # each rank receives the average (1 and 2 times (i + 1) -> 1.5 (i + 1)) of exactly its matrices
        assert res["owned"] == [i for i, o in enumerate(owners) if o == rank]
        for i, (lo, hi) in res["avg"].items():
            assert lo == hi == 1.5 * (i + 1)
        # auxiliary gradients are averaged in place on every rank
        assert res["aux"] == [(15.0, 15.0), (30.0, 30.0)]
        # every matrix's momentum (0.5 i, set by its owner) reaches every rank
        assert sorted(res["moms"]) == list(range(len(owners)))
        for i, (lo, hi) in res["moms"].items():
            assert lo == hi == 0.5 * i


def _sparse_worker(rank, world, port, results):
    """More ranks than matrices: some ranks own nothing."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = gpt_matrix_model(1, 8, 16)            # 6 matrices over 8 ranks
        opt = _StubOptimizer(model)
        sharding = MatrixSharding(opt, dist.group.WORLD, partition="lpt", copy_fn=_torch_copy)
        params = list(opt.named_matrices.values())
        for i, p in enumerate(params):
            p.grad = torch.full_like(p, float(i + 1) * (rank + 1))
        averaged = sharding.reduce_gradients([(p, p, {}) for p in params], [])
        send, recv, slots, unpack = sharding._layout()
        with torch.no_grad():
            for i, p in enumerate(params):
                if sharding.owns(p):
                    p.fill_(10.0 * i)
                    slots[id(p)].copy_(p)
            dist.all_gather_into_tensor(recv, send, group=dist.group.WORLD)
            for p, src in unpack:
                p.copy_(src.view_as(p))
        for i, p in enumerate(params):
            if sharding.owns(p):
                opt.state.setdefault(p, {})["momentum_buffer"] = torch.full_like(p, float(i))
        moms = sharding.consolidated_momentum()
        results[rank] = {"owned": sum(sharding.owns(p) for p in params),
                         "avg": sorted(float(v.mean()) for v in averaged.values()),
                         "weights": [float(p.mean()) for p in params],
                         "moms": sorted(float(v.mean()) for v in moms.values())}
    finally:
        dist.destroy_process_group()


def test_more_ranks_than_matrices():
    world = 8
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_sparse_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    owned = [results[r]["owned"] for r in range(world)]
    assert sum(owned) == 6 and owned.count(0) == 2
    mean_factor = sum(r + 1 for r in range(world)) / world        # 4.5
    for r in range(world):
        res = results[r]
        assert len(res["avg"]) == owned[r]
        assert all(any(abs(v - mean_factor * (i + 1)) < 1e-5 for i in range(6)) for v in res["avg"])
        assert res["weights"] == [10.0 * i for i in range(6)]      # every rank received every owner's matrix
        assert res["moms"] == [float(i) for i in range(6)]


def _skip_worker(rank, world, port, results):
    """exchange() with a matrix that has no gradient this step: its owner does
    not step it, and no rank may overwrite its weights from the stale slot."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = gpt_matrix_model(2, 16, 64)
        opt = _StubOptimizer(model)
        sharding = MatrixSharding(opt, dist.group.WORLD, partition="lpt", copy_fn=_torch_copy)
        params = list(opt.named_matrices.values())
        skipped = {0, 5}                      # e.g. an unused layer: grad None on every rank
        slots = sharding._layout()[2]
        history = []
        for step in range(2):
            stepped = [i for i in range(len(params)) if i not in skipped or step == 1]
            with torch.no_grad():
                if step == 0:
                    for i, p in enumerate(params):
                        p.fill_(-1.0 - i)     # the weights every rank starts from
                for i in stepped:
                    p = params[i]
                    if sharding.owns(p):      # test-only compute stub: the owner's update
                        p.fill_(100.0 * i + 10.0 * step + sharding.rank)
                        slots[id(p)].copy_(p)
            sharding.exchange([(params[i], params[i], {}) for i in stepped])
            history.append([float(p.min()) for p in params] + [float(p.max()) for p in params])
        results[rank] = {"history": history, "owners": [sharding.owner(p) for p in params]}
    finally:
        dist.destroy_process_group()


def test_exchange_keeps_weights_of_matrices_without_gradient():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_skip_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    r0, r1 = results[0], results[1]
    assert r0 == r1
    owners = r0["owners"]
    n = len(owners)
    assert {owners[0], owners[5]} <= {0, 1}
    for step, row in enumerate(r0["history"]):
        lo, hi = row[:n], row[n:]
        for i in range(n):
            if i in (0, 5) and step == 0:
                expected = -1.0 - i            # not stepped: every rank keeps its weights
            else:
                expected = 100.0 * i + 10.0 * step + owners[i]
            assert lo[i] == hi[i] == expected, (step, i, lo[i], hi[i], expected)


def test_unknown_transport_is_rejected():
    with pytest.raises(ValueError):
        MatrixSharding(None, None, transport="rdma")


def _transport_worker(rank, world, port, results):
    """The weight transport on a gloo group: "auto" keeps the NCCL-style
    all-gather (peer stores need CUDA buffers under NCCL), and "peer" fails on
    every rank together instead of leaving one rank in a collective."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        opt = _StubOptimizer(gpt_matrix_model(2, 16, 64))
        auto = MatrixSharding(opt, dist.group.WORLD, transport="auto")
        out = {"auto_peers": list(auto.peer_bases)}
        auto.close()  # nothing mapped: no collective, no error
        opt2 = _StubOptimizer(gpt_matrix_model(2, 16, 64))
        try:
            MatrixSharding(opt2, dist.group.WORLD, transport="peer")
            out["peer"] = "built"
        except RuntimeError as e:
            out["peer"] = "refused" if "transport='peer'" in str(e) else f"other: {e}"
        # the group is still usable after the refusal: the ranks stayed paired
        t = torch.ones(1)
        dist.all_reduce(t)
        out["after"] = float(t.item())
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_weight_transport_falls_back_or_refuses_together_on_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_transport_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        res = results[rank]
        assert res["auto_peers"] == [] and res["peer"] == "refused" and res["after"] == float(world), res
