"""ctypes binding of the C ABI in ``include/piper_b200.h`` (``libpiper_b200.so``).

The library is built in-tree by ``piper-kernels_b200/build.py`` (or
``__graft_entry__.build()``) into ``piper_kernels/_lib/``.  There is no
fallback: if the shared library is missing, every entry point raises
:class:`NativeLibraryMissing` with the build instructions.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "libpiper_b200.so"

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_DEVICE = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_WORKSPACE_TOO_SMALL = 5
FLOAT16 = 0
BFLOAT16 = 1
NO_ALLOC_WORKSPACE_BYTES = 16 * 1024 * 1024  # PIPER_B200_NO_ALLOC_WORKSPACE_BYTES
STATE_LOAD = 1  # PIPER_B200_STATE_LOAD
STATE_STORE = 2  # PIPER_B200_STATE_STORE

# Every symbol include/piper_b200.h declares (tests check the library exports them).
EXPORTED_SYMBOLS = (
    "piper_b200_abi_version",
    "piper_b200_last_error",
    "piper_b200_supports_device",
    "piper_b200_workspace_bytes",
    "piper_b200_workspace_layout",
    "piper_b200_prepass",
    "piper_b200_attention_prepared",
    "piper_b200_attention_fwd",
    "piper_b200_select_plan",
    "piper_b200_attention_prepared_plan",
    "piper_b200_attention_fwd_no_alloc",
    "piper_b200_shard_column_sums",
    "piper_b200_shard_prepass",
    "piper_b200_attention_shard",
    "piper_b200_attention_shard_range",
    "piper_b200_state_bytes",
    "piper_b200_host_scratch_bytes",
    "piper_b200_attention_fwd_host",
    "piper_b200_sage2pp_layout",
    "piper_b200_sage2pp_workspace_bytes",
    "piper_b200_sage2pp_prepass",
    "piper_b200_sage2pp_attention_prepared",
    "piper_b200_sage2pp_fwd",
    "piper_b200_device_status",
    "piper_b200_selftest_wait_timeout",
    "piper_b200_selftest_exp2",
    "piper_b200_selftest_gemm_i8",
)


class NativeLibraryMissing(RuntimeError):
    """The compiled sm_100a library is not present next to the package."""


class WorkspaceLayout(ctypes.Structure):
    """Mirror of ``piper_b200_workspace_layout_t``."""

    _fields_ = [
        (name, ctypes.c_uint64)
        for name in (
            "q8", "k8", "v8t", "qscale", "kscale", "vscale", "vlog2", "vrcp",
            "kmean", "vmean", "ksum", "vsum", "counter", "total_bytes",
        )
    ] + [(name, ctypes.c_int64) for name in ("q_groups", "k_groups", "nk_pad", "chunks")] + [
        (name, ctypes.c_uint64) for name in ("kv_pack", "kv_pack_bytes", "totals", "split_state")
    ] + [("split_units_max", ctypes.c_int64)]


class Plan(ctypes.Structure):
    """Mirror of ``piper_b200_plan_t``."""

    _fields_ = [(name, ctypes.c_int32) for name in ("tile_rows", "key_block", "stages", "rearm", "heavy_first",
                                                     "split_k")] + [
        (name, ctypes.c_int64) for name in ("tiles", "tail_tiles", "ctas")
    ] + [(name, ctypes.c_int32) for name in ("kernels", "sms")]


class Sage2ppLayout(ctypes.Structure):
    """Mirror of ``piper_b200_sage2pp_layout_t``."""

    _fields_ = [
        (name, ctypes.c_uint64)
        for name in (
            "q8", "qscale", "k8", "v8t", "kscale", "kmask", "vscale", "kmean", "ksum", "vmax", "counter",
            "total_bytes",
        )
    ] + [(name, ctypes.c_int64) for name in ("nk_pad", "chunks")]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_I64 = ctypes.c_int64
_STRIDES = ctypes.c_int64 * 3
_VP = ctypes.c_void_p


def _declare(lib: ctypes.CDLL) -> None:
    lib.piper_b200_abi_version.restype = ctypes.c_int
    lib.piper_b200_last_error.restype = ctypes.c_char_p
    lib.piper_b200_supports_device.argtypes = [ctypes.c_int]
    lib.piper_b200_supports_device.restype = ctypes.c_int
    lib.piper_b200_workspace_bytes.argtypes = [_I64] * 5 + [ctypes.POINTER(ctypes.c_size_t)]
    lib.piper_b200_workspace_bytes.restype = ctypes.c_int
    lib.piper_b200_workspace_layout.argtypes = [_I64] * 5 + [ctypes.POINTER(WorkspaceLayout)]
    lib.piper_b200_workspace_layout.restype = ctypes.c_int
    tensor3 = [_VP, _STRIDES] * 3
    lib.piper_b200_prepass.argtypes = tensor3 + [ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_prepass.restype = ctypes.c_int
    lib.piper_b200_attention_prepared.argtypes = [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_attention_prepared.restype = ctypes.c_int
    lib.piper_b200_attention_fwd.argtypes = tensor3 + [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_attention_fwd.restype = ctypes.c_int
    lib.piper_b200_select_plan.argtypes = [_I64] * 5 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(Plan)]
    lib.piper_b200_select_plan.restype = ctypes.c_int
    lib.piper_b200_attention_prepared_plan.argtypes = [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, ctypes.POINTER(Plan), _VP,
    ]
    lib.piper_b200_attention_prepared_plan.restype = ctypes.c_int
    lib.piper_b200_attention_fwd_no_alloc.argtypes = tensor3 + [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP,
    ]
    lib.piper_b200_attention_fwd_no_alloc.restype = ctypes.c_int
    lib.piper_b200_shard_column_sums.argtypes = [_VP, _STRIDES, _VP, _STRIDES, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_shard_column_sums.restype = ctypes.c_int
    lib.piper_b200_shard_prepass.argtypes = tensor3 + [ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_int, _I64, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_shard_prepass.restype = ctypes.c_int
    lib.piper_b200_attention_shard.argtypes = [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _I64, _VP, ctypes.c_size_t, _VP, _VP, ctypes.c_int, _VP,
    ]
    lib.piper_b200_attention_shard.restype = ctypes.c_int
    lib.piper_b200_attention_shard_range.argtypes = [_VP, ctypes.c_int] + [_I64] * 9 + [
        ctypes.c_double, ctypes.c_int, _I64, _VP, ctypes.c_size_t, _VP, _VP, ctypes.c_int, _VP,
    ]
    lib.piper_b200_attention_shard_range.restype = ctypes.c_int
    lib.piper_b200_state_bytes.argtypes = [_I64] * 4
    lib.piper_b200_state_bytes.restype = ctypes.c_size_t
    lib.piper_b200_host_scratch_bytes.argtypes = [_I64] * 5 + [ctypes.POINTER(ctypes.c_size_t)]
    lib.piper_b200_host_scratch_bytes.restype = ctypes.c_int
    lib.piper_b200_attention_fwd_host.argtypes = [_VP] * 4 + [ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_attention_fwd_host.restype = ctypes.c_int
    lib.piper_b200_sage2pp_layout.argtypes = [_I64] * 5 + [ctypes.POINTER(Sage2ppLayout)]
    lib.piper_b200_sage2pp_layout.restype = ctypes.c_int
    lib.piper_b200_sage2pp_workspace_bytes.argtypes = [_I64] * 5 + [ctypes.POINTER(ctypes.c_size_t)]
    lib.piper_b200_sage2pp_workspace_bytes.restype = ctypes.c_int
    lib.piper_b200_sage2pp_prepass.argtypes = tensor3 + [ctypes.c_int] + [_I64] * 5 + [_VP, ctypes.c_size_t, _VP]
    lib.piper_b200_sage2pp_prepass.restype = ctypes.c_int
    lib.piper_b200_sage2pp_attention_prepared.argtypes = [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_sage2pp_attention_prepared.restype = ctypes.c_int
    lib.piper_b200_sage2pp_fwd.argtypes = tensor3 + [_VP, ctypes.c_int] + [_I64] * 5 + [
        ctypes.c_double, ctypes.c_int, _VP, ctypes.c_size_t, _VP,
    ]
    lib.piper_b200_sage2pp_fwd.restype = ctypes.c_int
    lib.piper_b200_device_status.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]
    lib.piper_b200_device_status.restype = ctypes.c_int
    lib.piper_b200_selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_int), _VP]
    lib.piper_b200_selftest_wait_timeout.restype = ctypes.c_int
    lib.piper_b200_selftest_exp2.argtypes = [_VP, _VP, _VP, _I64, _VP]
    lib.piper_b200_selftest_exp2.restype = ctypes.c_int
    lib.piper_b200_selftest_gemm_i8.argtypes = [_VP, _VP, _VP] + [_I64] * 3 + [ctypes.c_int, _VP]
    lib.piper_b200_selftest_gemm_i8.restype = ctypes.c_int


def library() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryMissing(
                    f"{LIB_PATH} is missing: build the sm_100a extension with "
                    "`python piper-kernels_b200/build.py` (or __graft_entry__.build())"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            _declare(lib)
            _lib = lib
    return _lib


def last_error() -> str:
    return library().piper_b200_last_error().decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    """Raise the Python exception matching a piper_b200_status."""
    if status == OK:
        return
    message = f"{what}: {last_error()}"
    if status in (ERR_INVALID_ARGUMENT, ERR_WORKSPACE_TOO_SMALL):
        raise ValueError(message)
    if status == ERR_TIMEOUT:
        raise TimeoutError(message)
    raise RuntimeError(message)


def strides3(tensor) -> _STRIDES:
    s = tensor.stride()
    return _STRIDES(s[0], s[1], s[2])


def workspace_layout(batch: int, heads: int, nq: int, nk: int, d: int) -> WorkspaceLayout:
    layout = WorkspaceLayout()
    check(library().piper_b200_workspace_layout(batch, heads, nq, nk, d, ctypes.byref(layout)), "workspace layout")
    return layout


def sage2pp_layout(batch: int, heads: int, nq: int, nk: int, d: int) -> Sage2ppLayout:
    layout = Sage2ppLayout()
    check(library().piper_b200_sage2pp_layout(batch, heads, nq, nk, d, ctypes.byref(layout)), "sage2pp layout")
    return layout


def device_status(device: int, clear: bool = True) -> int:
    value = ctypes.c_uint32(0)
    check(library().piper_b200_device_status(device, 1 if clear else 0, ctypes.byref(value)), "device status")
    return int(value.value)
