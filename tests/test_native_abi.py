"""The C-ABI library loads and exports what include/piper_b200.h declares -- CPU only.

No compute call is made here (there is no GPU); only the pure host entry
points (layout arithmetic, argument checks that fail before any CUDA call).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from piper_kernels import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "piper_b200.h"


def _declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(piper_b200_\w+)\s*\(", text, flags=re.M))


def test_library_exports_every_declared_symbol() -> None:
    lib = _native.library()
    declared = _declared_symbols()
    assert declared == set(_native.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name


def test_abi_version() -> None:
    assert _native.library().piper_b200_abi_version() == 104


def test_workspace_layout_regions_are_aligned_and_disjoint() -> None:
    for shape in [(1, 1, 9, 11, 64), (2, 24, 4096, 4096, 128), (1, 40, 16384, 16384, 128), (2, 1, 200, 333, 128)]:
        b, h, nq, nk, d = shape
        L = _native.workspace_layout(*shape)
        bh = b * h
        regions = [
            (L.q8, bh * nq * d), (L.qscale, bh * L.q_groups * 4),
            (L.k8, bh * nk * d), (L.v8t, bh * d * L.nk_pad * 2), (L.kscale, bh * L.k_groups * 4),
            (L.vscale, bh * L.nk_pad * 4), (L.vlog2, bh * L.nk_pad * 4), (L.vrcp, bh * L.nk_pad * 4),
            (L.kmean, bh * d * 4), (L.vmean, bh * d * 4), (L.totals, 2 * bh * d * 8),
            (L.ksum, bh * L.chunks * d * 8), (L.vsum, bh * L.chunks * d * 8), (L.counter, bh * 4),
            (L.split_state, L.split_units_max * 256 * (d + 2) * 4),
        ]
        tiles = bh * -(-nq // 256)
        assert L.split_units_max == min(512, 8 * tiles)
        # The K/V pack is the contiguous span from the K codes to the end of vrcp.
        assert L.kv_pack == L.k8
        assert L.vrcp + bh * L.nk_pad * 4 <= L.kv_pack + L.kv_pack_bytes <= L.kmean
        assert L.q_groups == -(-nq // 32) and L.k_groups == -(-nk // 64)
        assert L.nk_pad % 64 == 0 and L.nk_pad >= nk
        end = 0
        for off, size in regions:
            assert off % 256 == 0 and off >= end
            end = off + size
        assert L.total_bytes >= end
        size = ctypes.c_size_t(0)
        _native.check(_native.library().piper_b200_workspace_bytes(b, h, nq, nk, d, ctypes.byref(size)), "bytes")
        assert size.value == L.total_bytes


def test_invalid_arguments_are_rejected_before_any_device_work() -> None:
    lib = _native.library()
    s = _native.strides3
    import torch

    q = torch.empty((1, 1, 8, 64), dtype=torch.float16)
    rc = lib.piper_b200_prepass(0, s(q), 0, s(q), 0, s(q), 7, 1, 1, 8, 8, 64, 0, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT
    assert "dtype" in _native.last_error()
    rc = lib.piper_b200_prepass(0, s(q), 0, s(q), 0, s(q), 0, 1, 1, 8, 8, 96, 0, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "head_dim" in _native.last_error()
    rc = lib.piper_b200_prepass(0, s(q), 0, s(q), 0, s(q), 0, 1, 1, 8, 9, 64, 1, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "causal" in _native.last_error()
    rc = lib.piper_b200_attention_prepared(0, 0, 1, 1, 8, 8, 64, float("nan"), 0, 1, 1, None)
    assert rc == _native.ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError, match="head_dim"):
        _native.check(lib.piper_b200_attention_fwd(0, s(q), 0, s(q), 0, s(q), 0, 0, 1, 1, 8, 8, 32, 0.1, 0, 0, 0, None), "fwd")


def test_shard_entry_points_check_arguments_on_the_host() -> None:
    lib = _native.library()
    s = _native.strides3
    import torch

    q = torch.empty((1, 1, 128, 64), dtype=torch.float16)
    assert lib.piper_b200_state_bytes(2, 3, 100, 64) == 2 * 3 * 100 * 66 * 4
    assert lib.piper_b200_state_bytes(0, 3, 100, 64) == 0
    rc = lib.piper_b200_shard_prepass(0, s(q), 0, s(q), 0, s(q), 0, 1, 1, 128, 128, 64, 0, 64, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "total_keys" in _native.last_error()
    rc = lib.piper_b200_attention_shard(0, 0, 1, 1, 128, 128, 64, 0.1, 0, 0, 0, 0, 0, 0, 4, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "state_mode" in _native.last_error()
    rc = lib.piper_b200_attention_shard(0, 0, 1, 1, 128, 128, 64, 0.1, 0, 64, 0, 0, 0, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "causal_shift" in _native.last_error()
    rc = lib.piper_b200_shard_column_sums(0, s(q), 0, s(q), 0, 1, 1, 128, 128, 64, 0, 0, 0, None)
    assert rc == _native.ERR_INVALID_ARGUMENT and "NULL" in _native.last_error()


def test_missing_library_fails_loudly(monkeypatch: pytest.MonkeyPatch, tmp_path: Path) -> None:
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "absent.so")
    with pytest.raises(_native.NativeLibraryMissing, match="build"):
        _native.library()
