"""Drop-in SandMuon optimizers whose arithmetic runs on the B200 CUDA engine.

Same constructor arguments, selection rule, q/k/v statistic sharing, hooks,
errors and state keys as the eager reference (sandmuon/optimizer.py:96-328);
every tensor operation of the hooks and of `step()` is a call into
libsandmuon_b200.so.  Models must live on an sm_100 GPU; there is no CPU path.
"""
from __future__ import annotations

import math
import re
from typing import Callable

import torch
from torch import nn
from torch.optim import Optimizer

from . import _lib, engine
from .coefficients import S8_COEFFICIENTS, S8_MARGIN, S8_MULTIPLIER
from .functional import (_graft_direction, _s8_fp32, diagonal_inverse_sqrt, rank1_inverse_sqrt,  # noqa: F401
                         rank1_mapback, rank1_whiten)

_QKV_SHARING = re.compile(r"^(transformer\.h\.\d+\.attn\.)[kv]_proj\.weight$")


class DiagonalWeightedPE(Optimizer):
    """SandMuon with diagonal whitening on both sides of each weight matrix.

    Each selected Linear weight is updated along the Schatten-8 polar
    direction of its Nesterov momentum, whitened on the input side by the
    running second moment of the layer's activations and on the output side
    by that of its output cotangents.  Those moments are summed by forward
    and cotangent hooks over all microbatches of a step, then folded into
    exponential averages (factor 0.97) at step().  Other trainable parameters
    take AdamW at a tenth of the learning rate with weight decay 0.01;
    momentum is 0.8.

    Extra keywords: `process_group` (torch.distributed group or None) shards
    the S8 work over the group's ranks, `partition` ("lpt" or "layer") picks
    the owners, `exchange` ("weights" or "bf16_delta") what the owners
    exchange, `transport` ("auto", "peer" or "nccl") how updated weights
    reach the other ranks (peer stores from the update kernel, or an NCCL
    all-gather), and `reduce_gradients=True` makes step() average the
    gradients over the group itself (reduce-scatter of the matrix gradients
    to their owners, all-reduce of the rest) in place of a data-parallel
    wrapper's all-reduce; see sandmuon_b200.distributed.
    """

    def __init__(self, model: nn.Module, lr: float, *, rank_one_a: bool = False,
                 module_filter: Callable[[str, nn.Module], bool] | None = None,
                 process_group=None, partition: str = "lpt", exchange: str = "weights",
                 reduce_gradients: bool = False, transport: str = "auto"):
        choose = module_filter or (lambda name, module: isinstance(module, nn.Linear))
        matrices: dict[str, nn.Parameter] = {}
        modules: dict[str, nn.Module] = {}
        for name, module in dict(model.named_modules()).items():
            if name and choose(name, module):
                parameter = getattr(module, "weight", None)
                if isinstance(parameter, nn.Parameter) and parameter.requires_grad and parameter.ndim == 2:
                    matrices[name + ".weight"] = parameter
                    modules[name + ".weight"] = module
        if not matrices:
            raise ValueError("No eligible trainable linear weights found")

        self.named_matrices = matrices
        self.parameter_names = {id(p): name for name, p in matrices.items()}
        self.rank_one_a = bool(rank_one_a)
        self.statistic_beta = .97
        self.s8_coefficients = S8_COEFFICIENTS
        self.s8_margin = S8_MARGIN
        self.s8_multiplier = S8_MULTIPLIER
        self._group_constants = {}

        # q/k/v sharing rule of the production run (sandmuon/optimizer.py:128-135)
        self.a_sources = {id(p): p for p in matrices.values()}
        for name, parameter in matrices.items():
            match = _QKV_SHARING.match(name)
            if match:
                q = matrices.get(match.group(1) + "q_proj.weight")
                if q is not None:
                    self.a_sources[id(parameter)] = q

        matrix_ids = {id(p) for p in matrices.values()}
        auxiliary = [p for p in model.parameters() if p.requires_grad and id(p) not in matrix_ids]
        defaults = dict(lr=float(lr), use_muon=True, momentum=.8, weight_decay=0.,
                        adamw_lr_ratio=.1, adamw_betas=(.9, .999), adamw_eps=1e-8)
        groups = [dict(params=list(matrices.values()), use_muon=True)]
        if auxiliary:
            groups.append(dict(params=auxiliary, use_muon=False, weight_decay=.01))
        super().__init__(groups, defaults)

        self._plans: dict[tuple, engine.StepPlan] = {}
        self._stat_flat: dict = {}
        self._work: dict[int, tuple] = {}
        self._sharding = None
        if reduce_gradients and process_group is None:
            raise ValueError("reduce_gradients=True needs a process_group")
        self._reduce_gradients = bool(reduce_gradients)
        if process_group is not None:
            from .distributed import MatrixSharding
            self._sharding = MatrixSharding(self, process_group, partition=partition, exchange=exchange,
                                            transport=transport)

        self.handles = []
        for name, module in modules.items():
            parameter = matrices[name]
            self.handles.append(module.register_forward_hook(
                self._capture(parameter, capture_a=self.a_sources[id(parameter)] is parameter)))

    # ------------------------------------------------------------- hooks

    def _capture(self, parameter, *, capture_a):
        def hook(module, inputs, output):
            if (not module.training or not torch.is_grad_enabled() or
                    not isinstance(output, torch.Tensor) or not output.requires_grad):
                return
            x = inputs[0].detach()
            rows = x.reshape(-1, x.shape[-1])
            state = self.state[parameter]
            if capture_a:
                if "a_sum" not in state:
                    state["a_sum"] = self._stat_slot(parameter, "a_sum", rows.shape[-1], rows.device)
                    state["a_count"] = 0
                    if self.rank_one_a:
                        state["a_first_sum"] = self._stat_slot(parameter, "a_first_sum", rows.shape[-1], rows.device)
                engine.accumulate_column_stats(rows, state["a_sum"],
                                               state["a_first_sum"] if self.rank_one_a else None)
                state["a_count"] += rows.shape[0]

            def cotangent_hook(gradient):
                delta = gradient.detach().reshape(-1, gradient.shape[-1])
                if "b_sum" not in state:
                    state["b_sum"] = self._stat_slot(parameter, "b_sum", delta.shape[-1], delta.device)
                    state["b_count"] = 0
                engine.accumulate_column_stats(delta, state["b_sum"])
                state["b_count"] += delta.shape[0]
                return gradient
            output.register_hook(cotangent_hook)
        return hook

    # ------------------------------------------------- statistic storage

    def _stat_slot(self, parameter, key, n, device):
        """A zeroed statistic vector for state[parameter][key]: a view into one
        flat per-device buffer holding every statistic sum of the optimizer, so
        a data-parallel step all-reduces them in place with one collective.
        Falls back to a fresh tensor for shapes the layout does not expect."""
        flat = self._stat_flat.get(device)
        if flat is None:
            layout, offset = {}, 0
            for p in self.named_matrices.values():
                d_out, d_in = p.shape
                if self.a_sources[id(p)] is p:
                    for k in ("a_sum", "a_first_sum") if self.rank_one_a else ("a_sum",):
                        layout[(id(p), k)] = (offset, d_in)
                        offset += d_in
                layout[(id(p), "b_sum")] = (offset, d_out)
                offset += d_out
            flat = (torch.zeros(offset, dtype=torch.float32, device=device), layout)
            self._stat_flat[device] = flat
        buf, layout = flat
        where = layout.get((id(parameter), key))
        if where is None or where[1] != n:
            return torch.zeros(n, dtype=torch.float32, device=device)
        view = buf[where[0]:where[0] + n]
        view.zero_()
        return view

    def _flat_statistics(self, device, stat_specs):
        """The flat buffer if every statistic sum of this step is a view of it
        and every selected matrix takes part, else None."""
        flat = self._stat_flat.get(device)
        if flat is None:
            return None
        buf, layout = flat
        lo, hi = buf.data_ptr(), buf.data_ptr() + buf.numel() * 4
        n_sums = sum(1 + (fs is not None) for _, _, fs, _, _ in stat_specs)
        if n_sums != len(layout):
            return None
        for _, s_, fs, _, _ in stat_specs:
            for t in (s_, fs):
                if t is not None and not (lo <= t.data_ptr() < hi):
                    return None
        return buf

    # -------------------------------------------------------------- step

    def _collect(self):
        """Active matrices / auxiliaries and the host-side statistic checks,
        raising exactly as the reference does and before any device work
        (sandmuon/optimizer.py:184-185, :211-212)."""
        matrix_items, auxiliary_items = [], []
        checked: dict[int, int] = {}
        for group in self.param_groups:
            for parameter in group["params"]:
                if parameter.grad is None:
                    continue
                if group.get("use_muon", True):
                    source = self.a_sources[id(parameter)]
                    if id(source) not in checked:
                        if self.state[source].get("a_count", 0) < 1:
                            raise RuntimeError(
                                f"Missing activation statistics: {self.parameter_names[id(source)]}")
                        checked[id(source)] = self.state[source]["a_count"]
                    count = checked[id(source)]
                    got = self.state[parameter].get("b_count", 0)
                    if got != count:
                        raise RuntimeError(
                            f"Missing or mismatched cotangent statistics: {self.parameter_names[id(parameter)]}; "
                            f"expected {count}, got {got}")
                    matrix_items.append((parameter, source, group))
                else:
                    auxiliary_items.append((parameter, group))
        return matrix_items, auxiliary_items

    # ------------------------------------------- parameter dtypes / layouts
    # The kernels read and write contiguous FP32.  Like the reference, which
    # steps in FP32 on `gradient.float()` and adds `direction.to(param.dtype)`
    # (sandmuon/optimizer.py:245-248, 281, 315), other dtypes and strided
    # tensors are accepted: a gradient is converted to a contiguous FP32 copy
    # for the step, and a parameter is stepped through a persistent FP32 work
    # copy whose update is then added to it in its own dtype.

    @staticmethod
    def _native(t: torch.Tensor) -> bool:
        return t.dtype == torch.float32 and t.is_contiguous()

    @staticmethod
    def _fp32_grad(g: torch.Tensor) -> torch.Tensor:
        return g if DiagonalWeightedPE._native(g) else g.detach().float().contiguous()

    def _work_copy(self, parameter) -> torch.Tensor:
        """The FP32 tensor the kernels update in place of `parameter`: the
        parameter itself when it is contiguous FP32, else a persistent work
        copy refreshed from it (apply with _apply_work_copy after the step)."""
        if self._native(parameter):
            return parameter
        if self._sharding is not None:
            raise TypeError("a sharded sandmuon_b200 optimizer needs contiguous float32 parameters; got "
                            f"{parameter.dtype} {'contiguous' if parameter.is_contiguous() else 'strided'}")
        pair = self._work.get(id(parameter))
        if pair is None or pair[0].shape != parameter.shape or pair[0].device != parameter.device:
            pair = (torch.empty(parameter.shape, dtype=torch.float32, device=parameter.device),
                    torch.empty(parameter.shape, dtype=torch.float32, device=parameter.device))
            self._work[id(parameter)] = pair
        work, before = pair
        work.copy_(parameter.detach())
        if parameter.dtype != torch.float32:
            before.copy_(work)
        return work

    def _apply_work_copy(self, parameter) -> None:
        if self._native(parameter):
            return
        work, before = self._work[id(parameter)]
        if parameter.dtype == torch.float32:
            parameter.detach().copy_(work)
        else:
            parameter.detach().add_((work - before).to(parameter.dtype))

    @torch.no_grad()
    def step(self, closure=None):
        if closure is None:
            loss = None
        else:
            with torch.enable_grad():
                loss = closure()
        matrix_items, auxiliary_items = self._collect()
        averaged = {}
        if self._reduce_gradients:
            averaged = self._sharding.reduce_gradients(matrix_items, [p for p, _ in auxiliary_items])
        self._step_auxiliary(auxiliary_items)
        if matrix_items:
            self._step_matrices(matrix_items, averaged)
        if self._sharding is not None:
            self._sharding.exchange(matrix_items)
        return loss

    def _step_auxiliary(self, auxiliary_items):
        by_hyper: dict[tuple, list] = {}
        converted = []
        for parameter, group in auxiliary_items:
            _lib.ensure_device(parameter.device)
            state = self.state[parameter]
            if "exp_avg" not in state:
                state["exp_avg"] = torch.zeros(parameter.shape, dtype=torch.float32, device=parameter.device)
                state["exp_avg_sq"] = torch.zeros(parameter.shape, dtype=torch.float32, device=parameter.device)
                state["step"] = 0
            for key in ("exp_avg", "exp_avg_sq"):
                if not self._native(state[key]):
                    state[key] = state[key].float().contiguous()
            state["step"] += 1
            b1, b2 = group["adamw_betas"]
            key = (group["lr"] * group["adamw_lr_ratio"], float(b1), float(b2), group["adamw_eps"],
                   group["weight_decay"], parameter.device)
            work = self._work_copy(parameter)
            if work is not parameter:
                converted.append(parameter)
            by_hyper.setdefault(key, []).append(engine.AdamItem(work, self._fp32_grad(parameter.grad),
                                                                state["exp_avg"], state["exp_avg_sq"], state["step"]))
        for (lr, b1, b2, eps, wd, _device), items in by_hyper.items():
            engine.adamw_multi(items, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd)
        for parameter in converted:
            self._apply_work_copy(parameter)

    @property
    def sharding(self):
        """The MatrixSharding of a process-group optimizer, else None."""
        return self._sharding

    def _owned(self, matrix_items):
        if self._sharding is None:
            return matrix_items
        return [item for item in matrix_items if self._sharding.owns(item[0])]

    def _step_matrices(self, matrix_items, averaged=None):
        """averaged: {id(p): gradient} replacing p.grad (the group-averaged
        gradients of the matrices this rank owns)."""
        averaged = averaged or {}
        device = matrix_items[0][0].device
        _lib.ensure_device(device)
        # statistics of every active source / target (finished on every rank)
        sources: dict[int, torch.Tensor] = {}
        for parameter, source, _ in matrix_items:
            sources.setdefault(id(source), source)
        stat_index: dict[tuple, int] = {}
        stat_specs, counts, ema_init = [], [], []
        kind_a = _lib.SM_STAT_A_RANK1 if self.rank_one_a else _lib.SM_STAT_A_DIAG
        for source in sources.values():
            st = self.state[source]
            init = "a_ema" not in st
            if init:
                st["a_ema"] = torch.empty_like(st["a_sum"])
                if self.rank_one_a:
                    st["a_mean_ema"] = torch.empty_like(st["a_sum"])
            stat_index[("a", id(source))] = len(stat_specs)
            stat_specs.append((kind_a, st["a_sum"], st.get("a_first_sum") if self.rank_one_a else None,
                               st["a_ema"], st.get("a_mean_ema") if self.rank_one_a else None))
            counts.append(st["a_count"])
            ema_init.append(init)
        owned = self._owned(matrix_items)
        for parameter, source, _ in matrix_items:
            st = self.state[parameter]
            init = "b_ema" not in st
            if init:
                st["b_ema"] = torch.empty_like(st["b_sum"])
            stat_index[("b", id(parameter))] = len(stat_specs)
            stat_specs.append((_lib.SM_STAT_B, st["b_sum"], None, st["b_ema"], None))
            counts.append(self.state[source]["a_count"])
            ema_init.append(init)
        mats, grads, lrs, converted = [], [], [], []
        for parameter, source, group in owned:
            if parameter.device != device:
                raise RuntimeError("sandmuon_b200 expects every selected matrix on one CUDA device")
            grad = self._fp32_grad(averaged.get(id(parameter), parameter.grad))
            st = self.state[parameter]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros(parameter.shape, dtype=torch.float32, device=parameter.device)
            elif not self._native(st["momentum_buffer"]):
                st["momentum_buffer"] = st["momentum_buffer"].float().contiguous()
            work = self._work_copy(parameter)
            if work is not parameter:
                converted.append(parameter)
            export = self._sharding.send_slot(parameter) if self._sharding is not None else None
            mats.append((work, st["momentum_buffer"], stat_index[("a", id(source))],
                         stat_index[("b", id(parameter))], export))
            grads.append(grad)
            lrs.append(group["lr"])
        momentum = float(owned[0][2]["momentum"]) if owned else .8
        key = (tuple((m[0].data_ptr(), m[1].data_ptr(), m[2], m[3], 0 if m[4] is None else m[4].data_ptr())
                     for m in mats),
               tuple((s[0],) + tuple(0 if t is None else t.data_ptr() for t in s[1:]) for s in stat_specs),
               momentum, self.statistic_beta)
        plan = self._plans.get(key)
        if plan is None:
            if len(self._plans) > 8:
                for old in self._plans.values():
                    old.close()
                self._plans.clear()
            export_mode = self._sharding.export_mode if self._sharding is not None else _lib.SM_EXPORT_WEIGHTS
            plan = engine.StepPlan(device, mats, stat_specs, statistic_beta=self.statistic_beta, momentum=momentum,
                                   export_mode=export_mode)
            self._plans[key] = plan
            if self._sharding is not None and self._sharding.peer_bases:
                plan.set_peers(*self._sharding.peer_target())
        device_counts = None
        if self._sharding is not None:
            flat = self._flat_statistics(device, stat_specs)
            if flat is not None:
                sums = [flat]
            else:
                sums = []
                for kind, s_, fs, _, _ in stat_specs:
                    sums.append(s_)
                    if fs is not None:
                        sums.append(fs)
            device_counts = self._sharding.reduce_statistics(sums, counts)
        plan.step(grads, lrs, counts, ema_init, device_counts=device_counts)
        for parameter in converted:
            self._apply_work_copy(parameter)
        # host-side counters follow the reference (sums are zeroed on the device)
        for source in sources.values():
            self.state[source]["a_count"] = 0
        for parameter, _, _ in matrix_items:
            self.state[parameter]["b_count"] = 0
        self._last_plan = plan

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        if self._sharding is not None:
            # momentum lives only with a matrix's owner (a consolidated
            # checkpoint carries every matrix's)
            for parameter in self.named_matrices.values():
                if not self._sharding.owns(parameter):
                    self.state.get(parameter, {}).pop("momentum_buffer", None)
        for plan in self._plans.values():
            plan.close()
        self._plans.clear()

    def consolidated_state_dict(self) -> dict:
        """state_dict() in the reference's layout on every rank of a sharded
        optimizer: the momentum buffer of each matrix, held only by its owner,
        is gathered from the owners (a collective: call on every rank).  A
        single-device optimizer returns state_dict()."""
        sd = self.state_dict()
        if self._sharding is None:
            return sd
        index = {id(p): i for i, p in enumerate(p for g in self.param_groups for p in g["params"])}
        for pid, momentum in self._sharding.consolidated_momentum().items():
            sd["state"].setdefault(index[pid], {})["momentum_buffer"] = momentum
        return sd

    def close(self):
        """Removes the hooks and frees the plans; a sharded optimizer that
        delivers weights by peer stores also unmaps its peers' buffers, after
        a barrier (a collective: call on every rank)."""
        for handle in self.handles:
            handle.remove()
        self.handles.clear()
        for plan in self._plans.values():
            plan.close()
        self._plans.clear()
        if self._sharding is not None:
            self._sharding.close()


class RankOneAWeightedPE(DiagonalWeightedPE):
    """SandMuon whose activation-side whitener also removes the activation
    mean: the input covariance is modelled as diagonal plus the rank-one
    outer product of the mean, inverted exactly (DiagonalWeightedPE with
    rank_one_a=True)."""

    def __init__(self, model: nn.Module, lr: float, *,
                 module_filter: Callable[[str, nn.Module], bool] | None = None,
                 process_group=None, partition: str = "lpt", exchange: str = "weights",
                 reduce_gradients: bool = False, split_sides: bool = False, transport: str = "auto"):
        super().__init__(model, lr, rank_one_a=True, module_filter=module_filter,
                         process_group=process_group, partition=partition, exchange=exchange,
                         reduce_gradients=reduce_gradients, transport=transport)
        # The historical option of that name (reproduction/odl/optim/
        # diagonal_weighted_pe.py:408-410, 500-543) applies the rank-one
        # whitening and mapback on the activation side only.  The engine's
        # kernels always do: the cotangent side has no rank-one term, and the
        # activation side's correction runs along d_in in either orientation.
        # Both settings therefore run the same kernels, with identical results.
        self.split_sides = bool(split_sides)
