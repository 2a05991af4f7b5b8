"""CPU oracle for ``piper_attention`` -- test infrastructure, never the product.

Python face of ``oracle/piper_oracle.c``, a plain-C restatement of the Piper
Kernels 0.2.1 portable reference
(``src/piper_kernels/attention/piper_attention/reference.py:22-118`` and
``src/piper_kernels/attention/kernels/qk_quantization/int8/sage/reference.py:61-108``,
``qk_quantization="per_warp"``).  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg import this module; they use it as the
checker.  The shipped operator never touches it.

Parity of this oracle with the reference is pinned by ``tests/test_oracle.py``
against ``tests/golden/*.npz``, which ``tests/golden/make_golden.py`` produced
by running the reference itself.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "piper_oracle.c"
LIBRARY = ORACLE_DIR / "libpiper_oracle.so"
QUERY_GROUP = 32
KEY_GROUP = 64

_F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_I8P = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_lib: ctypes.CDLL | None = None


def build(force: bool = False) -> Path:
    """Compile the oracle with IEEE semantics (no FMA contraction, no fast-math)."""
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        subprocess.run(
            [
                "gcc",
                "-O3",
                "-fPIC",
                "-shared",
                "-fopenmp",
                "-ffp-contract=off",
                "-fno-fast-math",
                "-o",
                str(LIBRARY),
                str(SOURCE),
                "-lm",
            ],
            check=True,
        )
    return LIBRARY


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        lib = ctypes.CDLL(str(LIBRARY))
        i64 = ctypes.c_int64
        lib.pk_sequence_mean.argtypes = [_F32P, i64, i64, i64, _F32P]
        lib.pk_sequence_mean.restype = None
        lib.pk_quantize_groups.argtypes = [_F32P, ctypes.c_void_p, i64, i64, i64, i64, _I8P, _F32P]
        lib.pk_quantize_groups.restype = None
        lib.pk_quantize_rows.argtypes = [_F32P, ctypes.c_void_p, i64, i64, i64, _I8P, _F32P]
        lib.pk_quantize_rows.restype = None
        lib.pk_attention.argtypes = [
            _I8P, _F32P, _I8P, _F32P, _I8P, _F32P, ctypes.c_void_p,
            i64, i64, i64, i64, ctypes.c_float, ctypes.c_int, _F32P,
        ]
        lib.pk_attention.restype = None
        lib.pk_attention_shard.argtypes = [
            _I8P, _F32P, _I8P, _F32P, _I8P, _F32P, ctypes.c_void_p,
            i64, i64, i64, i64, ctypes.c_float, ctypes.c_int, i64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
        ]
        lib.pk_attention_shard.restype = None
        _lib = lib
    return _lib


def set_threads(count: int) -> None:
    """Bound the OpenMP team used by the oracle (honoured at the next parallel region)."""
    os.environ["OMP_NUM_THREADS"] = str(count)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(ctypes.c_int(count))
    except OSError:
        pass


def _as_f32(x) -> np.ndarray:
    """Exact widening of an fp16/bf16 tensor (torch or numpy) to contiguous fp32."""
    if hasattr(x, "detach"):
        x = x.detach().to("cpu").float().contiguous().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def sequence_mean(x: np.ndarray) -> np.ndarray:
    """Per-(b,h) feature mean over the sequence, ``[B,H,N,D] -> [B,H,D]``."""
    x = _as_f32(x)
    b, h, n, d = x.shape
    out = np.empty((b, h, d), np.float32)
    _load().pk_sequence_mean(x, b * h, n, d, out)
    return out


def quantize_groups(x, group: int, mean: np.ndarray | None = None):
    """Per-``group``-row INT8 codes and fp32 scales (qk reference.py:61-77)."""
    x = _as_f32(x)
    b, h, n, d = x.shape
    groups = -(-n // group)
    codes = np.empty((b, h, n, d), np.int8)
    scales = np.empty((b, h, groups), np.float32)
    m = None if mean is None else np.ascontiguousarray(mean, np.float32)
    _load().pk_quantize_groups(x, _ptr(m), b * h, n, d, group, codes, scales)
    return codes, scales


def quantize_rows(x, mean: np.ndarray | None = None):
    """Per-key-row INT8 codes and fp32 scales (reference.py:22-32)."""
    x = _as_f32(x)
    b, h, n, d = x.shape
    codes = np.empty((b, h, n, d), np.int8)
    scales = np.empty((b, h, n), np.float32)
    m = None if mean is None else np.ascontiguousarray(mean, np.float32)
    _load().pk_quantize_rows(x, _ptr(m), b * h, n, d, codes, scales)
    return codes, scales


@dataclass
class Prepared:
    """Quantized operands, in the reference's own (un-transposed) layouts."""

    query_int8: np.ndarray  # [B,H,Nq,D]
    query_scale: np.ndarray  # [B,H,ceil(Nq/32)]
    key_int8: np.ndarray  # [B,H,Nk,D]
    key_scale: np.ndarray  # [B,H,ceil(Nk/64)]
    value_int8: np.ndarray  # [B,H,Nk,D]
    value_scale: np.ndarray  # [B,H,Nk]
    key_mean: np.ndarray  # [B,H,D]
    value_mean: np.ndarray | None  # [B,H,D] (None when causal)


def prepare(query, key, value, is_causal: bool, *, key_mean=None, value_mean=None) -> Prepared:
    """The quantization prepass: K smoothing, per-group Q/K, per-row V.

    ``key_mean`` / ``value_mean`` override the computed means, which lets a
    test compare codes bit for bit against another implementation's means.
    """
    q = _as_f32(query)
    k = _as_f32(key)
    v = _as_f32(value)
    km = sequence_mean(k) if key_mean is None else np.ascontiguousarray(key_mean, np.float32)
    vm = None
    if not is_causal:
        vm = sequence_mean(v) if value_mean is None else np.ascontiguousarray(value_mean, np.float32)
    q8, qs = quantize_groups(q, QUERY_GROUP)
    k8, ks = quantize_groups(k, KEY_GROUP, km)
    v8, vs = quantize_rows(v, vm)
    return Prepared(q8, qs, k8, ks, v8, vs, km, vm)


def attention_prepared(p: Prepared, scale: float, is_causal: bool) -> np.ndarray:
    """The fused recurrence on prepared operands; returns fp32 ``[B,H,Nq,D]``."""
    b, h, nq, d = p.query_int8.shape
    nk = p.key_int8.shape[2]
    out = np.empty((b, h, nq, d), np.float32)
    vm = None if p.value_mean is None else np.ascontiguousarray(p.value_mean, np.float32)
    _load().pk_attention(
        p.query_int8, p.query_scale, p.key_int8, p.key_scale, p.value_int8,
        p.value_scale, _ptr(vm), b * h, nq, nk, d, ctypes.c_float(scale),
        1 if is_causal else 0, out,
    )
    return out


STATE_LOAD = 1
STATE_STORE = 2


def attention_shard(query_side: Prepared, key_side: Prepared, scale: float, is_causal: bool, *,
                    causal_shift: int = 0, state: tuple[np.ndarray, np.ndarray] | None = None,
                    state_mode: int = 0) -> np.ndarray | None:
    """The recurrence over one key shard (pk_attention_shard).

    Q codes/scales and the V mean come from ``query_side``; K/V codes and
    scales from ``key_side``.  ``state`` = (numerator f32 [B,H,Nq,D],
    (max, denominator) f32 [B,H,Nq,2]) is read with STATE_LOAD and written with
    STATE_STORE; without STATE_STORE the fp32 output is returned.
    """
    b, h, nq, d = query_side.query_int8.shape
    nk = key_side.key_int8.shape[2]
    out = None if state_mode & STATE_STORE else np.empty((b, h, nq, d), np.float32)
    so, sml = state if state is not None else (None, None)
    for arr, shape in ((so, (b, h, nq, d)), (sml, (b, h, nq, 2))):
        if state_mode and (arr is None or arr.dtype != np.float32 or arr.shape != shape
                           or not arr.flags.c_contiguous):
            raise ValueError("state arrays must be contiguous float32 of the query shard's shape")
    vm = None if query_side.value_mean is None else np.ascontiguousarray(query_side.value_mean, np.float32)
    _load().pk_attention_shard(
        query_side.query_int8, query_side.query_scale, key_side.key_int8, key_side.key_scale,
        key_side.value_int8, key_side.value_scale, _ptr(vm), b * h, nq, nk, d, ctypes.c_float(scale),
        1 if is_causal else 0, int(causal_shift), _ptr(so), _ptr(sml), int(state_mode), _ptr(out),
    )
    return out


def piper_attention(query, key, value, scale: float | None = None, is_causal: bool = False,
                    *, key_mean=None, value_mean=None) -> tuple[np.ndarray, Prepared]:
    """Oracle forward: returns the fp32 output (cast it to the input dtype) and the prepass."""
    d = query.shape[-1]
    scale = d**-0.5 if scale is None else float(scale)
    p = prepare(query, key, value, is_causal, key_mean=key_mean, value_mean=value_mean)
    return attention_prepared(p, scale, is_causal), p


def piper_attention_torch(query, key, value, scale: float | None = None, is_causal: bool = False):
    """Oracle forward returning a CPU torch tensor in the input dtype."""
    import torch

    out, _ = piper_attention(query, key, value, scale, is_causal)
    return torch.from_numpy(out).to(query.dtype)
