"""Shared pytest set-up: import paths, the ``gpu`` marker, golden fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
for entry in (REPO / "piper-kernels_b200", REPO):
    if str(entry) not in sys.path:
        sys.path.insert(0, str(entry))

GOLDEN_DIR = REPO / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


def golden_cases() -> list[str]:
    """Piper Attention fixtures (tests/golden/make_golden.py)."""
    return sorted(p.stem for p in GOLDEN_DIR.glob("*.npz") if not p.stem.startswith("s2pp_"))


def sage_cases() -> list[str]:
    """SageAttention2++ fixtures (tests/golden/make_golden_sage2pp.py)."""
    return sorted(p.stem for p in GOLDEN_DIR.glob("s2pp_*.npz"))


def load_sage_golden(name: str) -> dict:
    """SageAttention2++ case: inputs in their dtype, everything else as torch tensors."""
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    dtype = torch.float16 if str(z["dtype"]) == "float16" else torch.bfloat16
    case = {k: torch.from_numpy(np.array(z[k])) for k in z.files if k not in ("dtype",)}
    for key in ("query", "key", "value"):
        case[key] = torch.from_numpy(z[key].copy()).view(dtype)
    case.update(dtype=dtype, scale=float(z["scale"]), is_causal=bool(z["is_causal"]))
    return case


def load_golden(name: str) -> dict:
    """Golden case as torch tensors (inputs in their fp16/bf16 dtype)."""
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    dtype = torch.float16 if str(z["dtype"]) == "float16" else torch.bfloat16

    def half(key: str) -> torch.Tensor:
        return torch.from_numpy(z[key].view(np.int16).copy()).view(dtype)

    case = {k: z[k] for k in z.files}
    case.update(
        dtype=dtype,
        query=half("query"),
        key=half("key"),
        value=half("value"),
        out=half("out"),
        scale=float(z["scale"]),
        is_causal=bool(z["is_causal"]),
    )
    return case


def require_b200() -> torch.device:
    """Device for GPU tests: a missing GPU skips, a wrong GPU fails loudly."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"GPU tests need an sm_100 device, got sm_{major}{minor}"
    return torch.device("cuda:0")
