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
    """S8 directions weighted by activation and output-cotangent diagonals.

    Statistics are accumulated from every forward/backward microbatch between
    optimizer steps. Defaults match the 103M run: beta=.97, Muon momentum=.8,
    S8 margin=1.35, auxiliary AdamW LR ratio=.1 and decay=.01.

    Extra keywords: `process_group` (torch.distributed group or None) shards
    the S8 work over the group's ranks, `partition` ("lpt" or "layer") picks
    the owners, `exchange` ("weights" or "bf16_delta") what the owners
    all-gather, and `reduce_gradients=True` makes step() average the
    gradients over the group itself (reduce-scatter of the matrix gradients
    to their owners, all-reduce of the rest) in place of a data-parallel
    wrapper's all-reduce; see sandmuon_b200.distributed.
    """

    def __init__(self, model: nn.Module, lr: float, *, rank_one_a: bool = False,
                 module_filter: Callable[[str, nn.Module], bool] | None = None,
                 process_group=None, partition: str = "lpt", exchange: str = "weights",
                 reduce_gradients: bool = False):
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
        self._sharding = None
        if reduce_gradients and process_group is None:
            raise ValueError("reduce_gradients=True needs a process_group")
        self._reduce_gradients = bool(reduce_gradients)
        if process_group is not None:
            from .distributed import MatrixSharding
            self._sharding = MatrixSharding(self, process_group, partition=partition, exchange=exchange)

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

    @staticmethod
    def _require(t: torch.Tensor, what: str):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise TypeError(f"sandmuon_b200 needs contiguous float32 {what}; got {t.dtype} "
                            f"{'contiguous' if t.is_contiguous() else 'strided'}")

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
        for parameter, group in auxiliary_items:
            _lib.ensure_device(parameter.device)
            self._require(parameter, "auxiliary parameters")
            self._require(parameter.grad, "auxiliary gradients")
            state = self.state[parameter]
            if "exp_avg" not in state:
                state["exp_avg"] = torch.zeros_like(parameter, dtype=torch.float32)
                state["exp_avg_sq"] = torch.zeros_like(parameter, dtype=torch.float32)
                state["step"] = 0
            state["step"] += 1
            b1, b2 = group["adamw_betas"]
            key = (group["lr"] * group["adamw_lr_ratio"], float(b1), float(b2), group["adamw_eps"],
                   group["weight_decay"], parameter.device)
            by_hyper.setdefault(key, []).append(engine.AdamItem(parameter, parameter.grad, state["exp_avg"],
                                                                state["exp_avg_sq"], state["step"]))
        for (lr, b1, b2, eps, wd, _device), items in by_hyper.items():
            engine.adamw_multi(items, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd)

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
        mats, grads, lrs = [], [], []
        for parameter, source, group in owned:
            if parameter.device != device:
                raise RuntimeError("sandmuon_b200 expects every selected matrix on one CUDA device")
            grad = averaged.get(id(parameter), parameter.grad)
            self._require(parameter, "matrix parameters")
            self._require(grad, "matrix gradients")
            st = self.state[parameter]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(parameter, dtype=torch.float32)
            export = self._sharding.send_slot(parameter) if self._sharding is not None else None
            mats.append((parameter, st["momentum_buffer"], stat_index[("a", id(source))],
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
        for handle in self.handles:
            handle.remove()
        self.handles.clear()
        for plan in self._plans.values():
            plan.close()
        self._plans.clear()


class RankOneAWeightedPE(DiagonalWeightedPE):
    """Production SAND variant with exact rank-one activation mean correction."""

    def __init__(self, model: nn.Module, lr: float, *,
                 module_filter: Callable[[str, nn.Module], bool] | None = None,
                 process_group=None, partition: str = "lpt", exchange: str = "weights",
                 reduce_gradients: bool = False):
        super().__init__(model, lr, rank_one_a=True, module_filter=module_filter,
                         process_group=process_group, partition=partition, exchange=exchange,
                         reduce_gradients=reduce_gradients)
