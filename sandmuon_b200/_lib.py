"""ctypes binding of libsandmuon_b200.so (declared in include/sandmuon_b200.h).

The library is the only compute path of this package: if it is missing or the
device is not an sm_100 GPU, every entry point raises instead of falling back.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# SANDMUON_B200_LIB names another build of the library (for example one
# compiled with different SMB_* tuning macros); default: the in-tree build.
LIB_PATH = Path(os.environ.get("SANDMUON_B200_LIB") or Path(__file__).resolve().parent / "libsandmuon_b200.so")

SM_OK = 0
SM_STAT_A_DIAG = 0
SM_STAT_A_RANK1 = 1
SM_STAT_B = 2
SM_EPI_F32 = 0
SM_EPI_BF16 = 1
SM_EPI_HILO = 2
SM_EPI_F32_NORM = 3
SM_EPI_POLY = 4
SM_EPI_POLY_HILO = 5
SM_EPI_SYMMETRIC = 0x100
SM_EPI_NORM_SLOTS = 16
SM_GEMM_B_KMAJOR = 1
SM_GEMM_A_MNMAJOR = 2
SM_GEMM_PAIR = 4
SM_GEMM_BN128 = 8
SM_EXPORT_WEIGHTS = 0
SM_EXPORT_BF16_DELTA = 1
SM_TCLASS_GEMM = 0
SM_TCLASS_ELEMWISE = 1
SM_TCLASS_STATS = 2
SM_TCLASS_COUNT = 3

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.float64: 3}

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float


class SmMatrixSpec(ctypes.Structure):
    _fields_ = [("weight", _c_void_p), ("momentum", _c_void_p), ("export_to", _c_void_p), ("d_out", _c_i32),
                ("d_in", _c_i32), ("a_stat", _c_i32), ("b_stat", _c_i32)]


class SmCopySpec(ctypes.Structure):
    _fields_ = [("dst", _c_void_p), ("src", _c_void_p), ("bytes", _c_i64)]


class SmStatSpec(ctypes.Structure):
    _fields_ = [("sum", _c_void_p), ("first_sum", _c_void_p), ("ema", _c_void_p), ("mean_ema", _c_void_p),
                ("n", _c_i32), ("kind", _c_i32)]


class SmPlanSpec(ctypes.Structure):
    _fields_ = [("matrices", ctypes.POINTER(SmMatrixSpec)), ("n_matrices", _c_i32),
                ("stats", ctypes.POINTER(SmStatSpec)), ("n_stats", _c_i32),
                ("statistic_beta", _c_float), ("momentum", _c_float), ("export_mode", _c_i32)]


class SmDeltaSpec(ctypes.Structure):
    _fields_ = [("weight", _c_void_p), ("delta", _c_void_p), ("numel", _c_i64)]


class SmStepArgs(ctypes.Structure):
    _fields_ = [("grads", ctypes.POINTER(_c_void_p)), ("lrs", ctypes.POINTER(_c_float)),
                ("counts", ctypes.POINTER(_c_i64)), ("ema_init", ctypes.POINTER(_c_i32)),
                ("device_counts", _c_void_p)]


class SmAdamTensor(ctypes.Structure):
    _fields_ = [("param", _c_void_p), ("grad", _c_void_p), ("exp_avg", _c_void_p), ("exp_avg_sq", _c_void_p),
                ("numel", _c_i64), ("bias_correction1", _c_float), ("bias_correction2", _c_float)]


# name -> (restype, argtypes); every symbol include/sandmuon_b200.h declares.
SIGNATURES = {
    "sm_version": (_c_int, []),
    "sm_last_error": (ctypes.c_char_p, []),
    "sm_init_device": (_c_int, []),
    "sm_device_status": (_c_int, [ctypes.POINTER(_c_int), _c_void_p]),
    "sm_stats_workspace_bytes": (_c_size, [_c_i64, _c_i64]),
    "sm_stats_accumulate": (_c_int, [_c_void_p, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_void_p, _c_void_p,
                                     _c_void_p, _c_size, _c_void_p]),
    "sm_stats_accumulate_noalloc": (_c_int, [_c_void_p, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_void_p,
                                             _c_void_p, _c_void_p]),
    "sm_plan_workspace_bytes": (_c_int, [ctypes.POINTER(SmPlanSpec), ctypes.POINTER(_c_size)]),
    "sm_plan_create": (_c_int, [ctypes.POINTER(SmPlanSpec), _c_void_p, _c_size, _c_void_p, ctypes.POINTER(_c_void_p)]),
    "sm_plan_step": (_c_int, [_c_void_p, ctypes.POINTER(SmStepArgs), _c_void_p]),
    "sm_plan_set_replay": (_c_int, [_c_void_p, _c_int]),
    "sm_plan_set_peers": (_c_int, [_c_void_p, _c_void_p, _c_i64, ctypes.POINTER(_c_void_p), _c_i32]),
    "sm_ipc_export": (_c_int, [_c_void_p, _c_void_p, ctypes.POINTER(_c_i64)]),
    "sm_ipc_open": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "sm_ipc_close": (_c_int, [_c_void_p]),
    "sm_plan_set_timing": (_c_int, [_c_void_p, _c_int]),
    "sm_plan_timing_read": (_c_int, [_c_void_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_c_i64),
                                     ctypes.POINTER(ctypes.c_double)]),
    "sm_plan_launches_per_step": (_c_int, [_c_void_p, ctypes.POINTER(_c_i64)]),
    "sm_plan_destroy": (_c_int, [_c_void_p]),
    "sm_copy_multi": (_c_int, [ctypes.POINTER(SmCopySpec), _c_i32, _c_void_p]),
    "sm_s8_workspace_bytes": (_c_size, [_c_i32, _c_i32, _c_i32]),
    "sm_s8_polar": (_c_int, [_c_void_p, _c_void_p, _c_i32, _c_i32, _c_i32, _c_void_p, _c_size, _c_void_p]),
    "sm_apply_bf16_delta_multi": (_c_int, [ctypes.POINTER(SmDeltaSpec), _c_i32, _c_void_p]),
    "sm_s8_executed_flops": (_c_int, [_c_i32, _c_i32, _c_i32, ctypes.POINTER(ctypes.c_double)]),
    "sm_adamw_multi": (_c_int, [ctypes.POINTER(SmAdamTensor), _c_i32, _c_float, _c_float, _c_float, _c_float,
                                _c_float, _c_void_p]),
    "sm_gemm_bf16": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_i32, _c_i32, _c_i32, _c_i32,
                              _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_float, _c_float,
                              _c_float, _c_void_p, _c_void_p]),
}

_lib = None
_lib_lock = threading.Lock()
_devices_ready: set[int] = set()


def load() -> ctypes.CDLL:
    """Loads the shared library once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"sandmuon_b200: {LIB_PATH.name} is not built; run `python -m sandmuon_b200.csrc.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().sm_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != SM_OK:
        raise RuntimeError(f"sandmuon_b200 {what} failed (status {rc}): {last_error()}")


def ensure_device(device: torch.device) -> None:
    """Verifies `device` is a CUDA sm_100 GPU the library can run on."""
    if device.type != "cuda":
        raise RuntimeError(f"sandmuon_b200 runs on CUDA (sm_100) tensors only; got a tensor on {device}")
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index in _devices_ready:
        return
    with torch.cuda.device(index):
        check(load().sm_init_device(), "device check")
    _devices_ready.add(index)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


IPC_HANDLE_BYTES = 64


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(CUDA IPC handle of the allocation holding t, t's byte offset in it)."""
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    offset = _c_i64(0)
    with torch.cuda.device(t.device):
        check(load().sm_ipc_export(_c_void_p(t.data_ptr()), handle, ctypes.byref(offset)), "IPC export")
    return handle.raw, offset.value


def ipc_open(handle: bytes, device: torch.device) -> int:
    """Maps another process's exported allocation into `device`'s address
    space (peer access); returns the mapped base address."""
    base = _c_void_p(0)
    buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        check(load().sm_ipc_open(buf, ctypes.byref(base)), "IPC open")
    return int(base.value)


def ipc_close(base: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        check(load().sm_ipc_close(_c_void_p(base)), "IPC close")


def device_status(device: torch.device) -> int:
    """Reads and clears the library's device-side timeout word (synchronises)."""
    status = _c_int(0)
    with torch.cuda.device(device):
        check(load().sm_device_status(ctypes.byref(status), _c_void_p(stream_handle(device))), "device status")
    return status.value
