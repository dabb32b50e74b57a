"""Python-facing wrappers of the CUDA engine (libsandmuon_b200.so).

Each function validates its tensors on the host (device, dtype, layout), then
makes one C-ABI call on the tensor's current CUDA stream.  PyTorch only
allocates memory here; all arithmetic happens in the library's kernels.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(_lib.stream_handle(device))


# ----------------------------------------------------------------- workspaces

class _Workspaces:
    """Grow-only byte buffers keyed by (device, stream, tag).

    Buffers are reused in stream order, so a buffer is never shared by two
    streams; the caching allocator keeps a replaced buffer alive until the
    work already queued on that stream has consumed it."""

    def __init__(self):
        self._buffers: dict[tuple, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
        key = (device.index, _lib.stream_handle(device), tag)
        buf = self._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._buffers[key] = buf
        return buf


_workspaces = _Workspaces()


# ----------------------------------------------------------- N1: statistics

def accumulate_column_stats(rows: torch.Tensor, sum_sq: torch.Tensor, total: torch.Tensor | None = None) -> None:
    """sum_sq += (rows.float()**2).sum(0); total += rows.float().sum(0).

    The CUDA replacement of the forward / cotangent hook reductions
    (sandmuon/optimizer.py:156-168, :170-178).  `rows` is a 2-D view in any of
    float32 / bfloat16 / float16 / float64 with arbitrary strides."""
    if rows.dim() != 2:
        raise ValueError("rows must be 2-D [n_rows, n_cols]")
    device = rows.device
    _lib.ensure_device(device)
    if rows.dtype not in _lib.DTYPE_CODES:
        raise TypeError(f"unsupported statistic input dtype {rows.dtype}")
    for acc in (sum_sq, total):
        if acc is not None and (acc.dtype != torch.float32 or acc.device != device or not acc.is_contiguous()
                                or acc.numel() != rows.shape[1]):
            raise ValueError("statistic accumulators must be contiguous float32 [n_cols] on the input device")
    n_rows, n_cols = rows.shape
    if n_rows == 0 or n_cols == 0:
        return
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = lib.sm_stats_workspace_bytes(n_rows, n_cols)
        ws = _workspaces.get(device, nbytes, "stats")
        rc = lib.sm_stats_accumulate(_ptr(rows), _lib.DTYPE_CODES[rows.dtype], n_rows, n_cols, rows.stride(0),
                                     rows.stride(1), _ptr(sum_sq), _ptr(total), _ptr(ws), ws.numel(), _stream(device))
    _lib.check(rc, "sm_stats_accumulate")


# ---------------------------------------------------------------- S8 (batch)

def s8_polar(x: torch.Tensor) -> torch.Tensor:
    """The engine's S8 polar map on a CUDA float32 [.., rows, cols] tensor.

    Same orientation, normalisation, coefficients and margin as _s8_fp32
    (sandmuon/optimizer.py:69-93); stages 1-4 run in compensated BF16 (hi/lo
    operand planes, three products) and stage 5 in BF16 on tcgen05 tensor
    cores, all with FP32 accumulation."""
    if x.dim() < 2:
        raise ValueError("s8_polar expects [..., rows, cols]")
    if x.dtype != torch.float32:
        raise TypeError("s8_polar expects float32 input")
    device = x.device
    _lib.ensure_device(device)
    rows, cols = x.shape[-2:]
    flat = x.reshape(-1, rows, cols).contiguous()
    batch = flat.shape[0]
    out = torch.empty_like(flat)
    if batch == 0 or rows == 0 or cols == 0:
        return out.reshape(x.shape)
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = lib.sm_s8_workspace_bytes(batch, rows, cols)
        ws = _workspaces.get(device, nbytes, "s8")
        rc = lib.sm_s8_polar(_ptr(flat), _ptr(out), batch, rows, cols, _ptr(ws), ws.numel(), _stream(device))
    _lib.check(rc, "sm_s8_polar")
    return out.reshape(x.shape)


def s8_executed_flops(batch: int, rows: int, cols: int, device=None) -> float:
    """Tensor-core FLOPs s8_polar executes for a [batch, rows, cols] input on
    `device` (computed tiles only; three products in compensated stages)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _lib.ensure_device(device)
    out = ctypes.c_double(0.0)
    with torch.cuda.device(device):
        rc = _lib.load().sm_s8_executed_flops(int(batch), int(rows), int(cols), ctypes.byref(out))
    _lib.check(rc, "sm_s8_executed_flops")
    return out.value


# ---------------------------------------------------------------- GEMM (tests)

def gemm_bf16(a_hi, b_hi, *, a_lo=None, b_lo=None, b_kmajor=True, a_mnmajor=False, pair=False, bn128=False,
              epilogue=_lib.SM_EPI_F32, out0=None, out1=None, alpha=None, aux=None, aux_lo=None,
              poly=(0.0, 0.0, 0.0), partials=None):
    """Direct access to the batched tcgen05 GEMM for unit tests.

    a: [batch, M, K] bf16, or [batch, K, M] (a_mnmajor); b: [batch, N, K]
    (b_kmajor) or [batch, K, N] bf16.  pair: 256-row tiles computed by CTA
    pairs (tcgen05 cta_group::2), M % 256 == 0.  bn128: 128-column tiles."""
    if a_mnmajor:
        batch, k, m = a_hi.shape
    else:
        batch, m, k = a_hi.shape
    n = b_hi.shape[1] if b_kmajor else b_hi.shape[2]
    layout = ((_lib.SM_GEMM_B_KMAJOR if b_kmajor else 0) | (_lib.SM_GEMM_A_MNMAJOR if a_mnmajor else 0)
              | (_lib.SM_GEMM_PAIR if pair else 0) | (_lib.SM_GEMM_BN128 if bn128 else 0))
    device = a_hi.device
    _lib.ensure_device(device)
    with torch.cuda.device(device):
        rc = _lib.load().sm_gemm_bf16(_ptr(a_hi), _ptr(a_lo), _ptr(b_hi), _ptr(b_lo), layout, batch, m, n, k,
                                      epilogue, _ptr(out0), _ptr(out1), _ptr(alpha), _ptr(aux), _ptr(aux_lo),
                                      float(poly[0]),
                                      float(poly[1]), float(poly[2]), _ptr(partials), _stream(device))
    _lib.check(rc, "sm_gemm_bf16")


# -------------------------------------------------------------------- AdamW

@dataclass
class AdamItem:
    param: torch.Tensor
    grad: torch.Tensor
    exp_avg: torch.Tensor
    exp_avg_sq: torch.Tensor
    step: int


def adamw_multi(items: list[AdamItem], *, lr: float, beta1: float, beta2: float, eps: float,
                weight_decay: float) -> None:
    """One fused multi-tensor AdamW update (sandmuon/optimizer.py:268-281)."""
    if not items:
        return
    device = items[0].param.device
    _lib.ensure_device(device)
    arr = (_lib.SmAdamTensor * len(items))()
    for slot, it in zip(arr, items):
        for t in (it.param, it.grad, it.exp_avg, it.exp_avg_sq):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device != device:
                raise TypeError("AdamW tensors must be contiguous float32 CUDA tensors on one device")
        slot.param = it.param.data_ptr()
        slot.grad = it.grad.data_ptr()
        slot.exp_avg = it.exp_avg.data_ptr()
        slot.exp_avg_sq = it.exp_avg_sq.data_ptr()
        slot.numel = it.param.numel()
        slot.bias_correction1 = 1.0 - beta1 ** it.step
        slot.bias_correction2 = 1.0 - beta2 ** it.step
    decay = 1.0 - lr * weight_decay
    with torch.cuda.device(device):
        rc = _lib.load().sm_adamw_multi(arr, len(items), lr, beta1, beta2, eps, decay, _stream(device))
    _lib.check(rc, "sm_adamw_multi")


# --------------------------------------------------------------------- plan

class StepPlan:
    """A native step plan over a fixed set of matrices and statistics.

    Holds the C++ SmPlan and the torch workspace it was carved from; the plan
    records raw pointers, so it must be rebuilt whenever any tensor it names
    is replaced (the optimizer keys plans by those pointers)."""

    def __init__(self, device: torch.device, matrices: list[tuple], stats: list[tuple], *,
                 statistic_beta: float, momentum: float, export_mode: int = _lib.SM_EXPORT_WEIGHTS):
        """matrices: (weight, momentum_buffer, a_stat_index, b_stat_index, export | None)
        stats: (kind, sum, first_sum | None, ema, mean_ema | None).
        export_mode: what the step writes to each export tensor, FP32 updated
        weights (SM_EXPORT_WEIGHTS) or BF16 update deltas (SM_EXPORT_BF16_DELTA)."""
        _lib.ensure_device(device)
        self.device = device
        self._keep = []
        mat_arr = (_lib.SmMatrixSpec * len(matrices))()
        for slot, (w, m, ia, ib, ex) in zip(mat_arr, matrices):
            slot.weight, slot.momentum = w.data_ptr(), m.data_ptr()
            slot.export_to = 0 if ex is None else ex.data_ptr()
            if ex is not None:
                self._keep.append(ex)
            slot.d_out, slot.d_in = w.shape
            slot.a_stat, slot.b_stat = ia, ib
            self._keep += [w, m]
        stat_arr = (_lib.SmStatSpec * len(stats))()
        for slot, (kind, s, fs, ema, mema) in zip(stat_arr, stats):
            slot.sum, slot.ema = s.data_ptr(), ema.data_ptr()
            slot.first_sum = fs.data_ptr() if fs is not None else 0
            slot.mean_ema = mema.data_ptr() if mema is not None else 0
            slot.n, slot.kind = s.numel(), kind
            self._keep += [s, ema] + [t for t in (fs, mema) if t is not None]
        self._spec = _lib.SmPlanSpec(mat_arr, len(matrices), stat_arr, len(stats), statistic_beta, momentum,
                                     export_mode)
        self._arrays = (mat_arr, stat_arr)
        lib = _lib.load()
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.sm_plan_workspace_bytes(ctypes.byref(self._spec), ctypes.byref(nbytes)), "plan layout")
        self.workspace = torch.empty(nbytes.value, dtype=torch.uint8, device=device)
        if self.workspace.data_ptr() % 256:
            raise RuntimeError("plan workspace is not 256-byte aligned")
        handle = ctypes.c_void_p(0)
        with torch.cuda.device(device):
            _lib.check(lib.sm_plan_create(ctypes.byref(self._spec), _ptr(self.workspace), nbytes.value,
                                          _stream(device), ctypes.byref(handle)), "sm_plan_create")
        self._handle = handle
        self.n_matrices = len(matrices)
        self.n_stats = len(stats)
        self._grads = (ctypes.c_void_p * self.n_matrices)()
        self._lrs = (ctypes.c_float * self.n_matrices)()
        self._counts = (ctypes.c_int64 * self.n_stats)()
        self._init = (ctypes.c_int32 * self.n_stats)()

    def step(self, grads: list[torch.Tensor], lrs: list[float], counts: list[int], ema_init: list[bool],
             device_counts: torch.Tensor | None = None) -> None:
        """device_counts: optional int64 CUDA tensor [n_stats] whose values replace
        `counts` on the device (all-reduced counts, no host synchronisation)."""
        for i, g in enumerate(grads):
            self._grads[i] = g.data_ptr()
            self._lrs[i] = lrs[i]
        for i, (c, e) in enumerate(zip(counts, ema_init)):
            self._counts[i] = c
            self._init[i] = 1 if e else 0
        if device_counts is not None and (device_counts.dtype != torch.int64 or device_counts.numel() != self.n_stats
                                          or device_counts.device != self.device):
            raise ValueError("device_counts must be an int64 tensor [n_stats] on the plan's device")
        args = _lib.SmStepArgs(self._grads, self._lrs, self._counts, self._init,
                               0 if device_counts is None else device_counts.data_ptr())
        with torch.cuda.device(self.device):
            rc = _lib.load().sm_plan_step(self._handle, ctypes.byref(args), _stream(self.device))
        _lib.check(rc, "sm_plan_step")

    def set_replay(self, enabled: bool) -> None:
        """Graph replay of the step's launches (on by default; identical results)."""
        _lib.check(_lib.load().sm_plan_set_replay(self._handle, int(enabled)), "sm_plan_set_replay")

    def set_peers(self, local_base: int, nbytes: int, peer_bases: list[int]) -> None:
        """From the next step on, every weight this plan updates inside
        [local_base, local_base + nbytes) is also stored at the same offset
        from each peer base (other ranks' copies of the flat weight buffer,
        mapped into this device); an empty list turns it off."""
        arr = (ctypes.c_void_p * max(1, len(peer_bases)))(*peer_bases)
        rc = _lib.load().sm_plan_set_peers(self._handle, ctypes.c_void_p(local_base), nbytes, arr, len(peer_bases))
        _lib.check(rc, "sm_plan_set_peers")

    def set_timing(self, enabled: bool) -> None:
        _lib.check(_lib.load().sm_plan_set_timing(self._handle, int(enabled)), "sm_plan_set_timing")

    def read_timing(self) -> dict:
        ms = (ctypes.c_double * _lib.SM_TCLASS_COUNT)()
        n = (ctypes.c_int64 * _lib.SM_TCLASS_COUNT)()
        flops = ctypes.c_double(0)
        _lib.check(_lib.load().sm_plan_timing_read(self._handle, ms, n, ctypes.byref(flops)), "sm_plan_timing_read")
        names = ("gemm", "elementwise", "stats")
        return {"ms": dict(zip(names, list(ms))), "launches": dict(zip(names, list(n))), "gemm_flops": flops.value}

    def launches_per_step(self) -> int:
        out = ctypes.c_int64(0)
        _lib.check(_lib.load().sm_plan_launches_per_step(self._handle, ctypes.byref(out)), "launch count")
        return out.value

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.load().sm_plan_destroy(self._handle)
            self._handle = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def copy_multi(pairs: list[tuple[torch.Tensor, torch.Tensor]], device: torch.device) -> None:
    """dst.copy_(src) for every (dst, src) pair of same-size contiguous CUDA
    tensors, in one kernel launch per 64 pairs."""
    if not pairs:
        return
    arr = (_lib.SmCopySpec * len(pairs))()
    for slot, (dst, src) in zip(arr, pairs):
        if dst.numel() * dst.element_size() != src.numel() * src.element_size():
            raise ValueError("copy_multi: size mismatch")
        slot.dst, slot.src, slot.bytes = dst.data_ptr(), src.data_ptr(), dst.numel() * dst.element_size()
    with torch.cuda.device(device):
        rc = _lib.load().sm_copy_multi(arr, len(pairs), _stream(device))
    _lib.check(rc, "sm_copy_multi")


def apply_bf16_delta_multi(pairs: list[tuple[torch.Tensor, torch.Tensor]], device: torch.device) -> None:
    """weight -= delta.float() for every (FP32 weight, BF16 delta) pair of
    contiguous CUDA tensors with equal element counts, in one kernel launch per
    64 pairs."""
    if not pairs:
        return
    arr = (_lib.SmDeltaSpec * len(pairs))()
    for slot, (w, d) in zip(arr, pairs):
        if w.dtype != torch.float32 or d.dtype != torch.bfloat16 or w.numel() != d.numel():
            raise ValueError("apply_bf16_delta_multi: needs float32 weights and bfloat16 deltas of equal size")
        slot.weight, slot.delta, slot.numel = w.data_ptr(), d.data_ptr(), w.numel()
    with torch.cuda.device(device):
        rc = _lib.load().sm_apply_bf16_delta_multi(arr, len(pairs), _stream(device))
    _lib.check(rc, "sm_apply_bf16_delta_multi")
