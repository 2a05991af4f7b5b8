"""Accelerator facts used to pick the backend.

Same shape as the reference's ``AcceleratorTarget``
(Piper Kernels 0.2.1, ``src/piper_kernels/_triton/targets.py:16-109``): plain
frozen data that policy code and tests can build without a GPU.  The B200
backend needs CUDA compute capability 10.0 exactly (``sm_100``): its kernels
are compiled for ``sm_100a`` and issue ``tcgen05`` instructions.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True, slots=True)
class AcceleratorTarget:
    backend: str
    architecture: str | None = None
    # Streaming multiprocessors: the launch plan sizes its waves by it (148 on a
    # B200; tests build targets with other counts).
    multi_processor_count: int | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "backend", self.backend.strip().lower())
        arch = None if self.architecture is None else str(self.architecture).strip().lower().partition(":")[0]
        object.__setattr__(self, "architecture", arch or None)

    @classmethod
    def from_device(cls, device: torch.device) -> "AcceleratorTarget":
        if device.type != "cuda":
            return cls(backend=device.type)
        if getattr(torch.version, "hip", None) is not None:
            return cls(backend="hip", architecture=getattr(torch.cuda.get_device_properties(device), "gcnArchName", None))
        major, minor = torch.cuda.get_device_capability(device)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        return cls(backend="cuda", architecture=f"sm{major}{minor}", multi_processor_count=sms)

    @property
    def cuda_capability(self) -> tuple[int, int] | None:
        if self.backend != "cuda" or self.architecture is None:
            return None
        digits = self.architecture.removeprefix("sm")
        if digits == self.architecture or not digits.isdecimal():
            return None
        return divmod(int(digits), 10)

    @property
    def supports_tcgen05_int8(self) -> bool:
        """True for sm_100 (B200-class): tcgen05.mma kind::i8 with TMEM accumulators."""
        return self.cuda_capability == (10, 0)

    @property
    def supports_tcgen05_fp8(self) -> bool:
        """True for sm_100 (B200-class): tcgen05.mma kind::f8f6f4 (FP8 e4m3) with TMEM accumulators."""
        return self.cuda_capability == (10, 0)
