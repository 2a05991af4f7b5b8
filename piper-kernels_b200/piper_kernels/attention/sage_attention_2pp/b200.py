"""B200 backend of SageAttention2++: custom op over the sm_100a C ABI.

Replaces the reference's Triton backend
(Piper Kernels 0.2.1, ``src/piper_kernels/attention/sage_attention_2pp/triton.py``):

* ``torch.ops.piper_kernels.sage_attention_2pp(query, key, value, scale, is_causal)``
  is registered with the same name, schema and fake implementation
  (triton.py:1135-1155);
* ``prepare_sage_attention_2pp`` / ``launch_sage_attention_2pp`` reproduce the
  reference's prepare/launch split (triton.py:1000-1102);
* device memory (output and one workspace holding every intermediate) comes
  from torch's caching allocator on the query's device; the kernels run on
  the current torch stream of that device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ... import _native

_DTYPE_CODES = {torch.float16: _native.FLOAT16, torch.bfloat16: _native.BFLOAT16}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass(frozen=True)
class PreparedSageAttention2pp:
    """Workspace of one call plus typed views of its intermediates.

    Scales are stored expanded: one Q scale per query row (the scale of the
    row's interleaved group) and one K scale per key; V codes are FP8 e4m3
    bytes stored transposed ``[B,H,D,Nk_pad]``.
    """

    workspace: torch.Tensor
    layout: _native.Sage2ppLayout
    shape: tuple[int, int, int, int, int]  # B, H, Nq, Nk, D
    dtype: torch.dtype
    is_causal: bool

    def _view(self, offset: int, count: int, dtype: torch.dtype, shape: tuple[int, ...]) -> torch.Tensor:
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return self.workspace[offset : offset + nbytes].view(dtype).view(shape)

    @property
    def query_int8(self) -> torch.Tensor:
        b, h, nq, _nk, d = self.shape
        return self._view(self.layout.q8, b * h * nq * d, torch.int8, (b, h, nq, d))

    @property
    def query_scale(self) -> torch.Tensor:
        """``[B,H,Nq]``: the per_thread group scale of each query row."""
        b, h, nq, _nk, _d = self.shape
        return self._view(self.layout.qscale, b * h * nq, torch.float32, (b, h, nq))

    @property
    def key_int8(self) -> torch.Tensor:
        b, h, _nq, nk, d = self.shape
        return self._view(self.layout.k8, b * h * nk * d, torch.int8, (b, h, nk, d))

    @property
    def key_scale(self) -> torch.Tensor:
        """``[B,H,Nk]``: the per_thread group scale of each key row."""
        b, h, _nq, nk, _d = self.shape
        pad = self.layout.nk_pad
        return self._view(self.layout.kscale, b * h * pad, torch.float32, (b, h, pad))[..., :nk]

    @property
    def value_fp8_transposed(self) -> torch.Tensor:
        """``[B,H,D,Nk_pad]`` FP8 e4m3 codes (padded keys are zero)."""
        b, h, _nq, _nk, d = self.shape
        pad = self.layout.nk_pad
        return self._view(self.layout.v8t, b * h * d * pad, torch.uint8, (b, h, d, pad)).view(torch.float8_e4m3fn)

    @property
    def value_fp8(self) -> torch.Tensor:
        """V codes in the reference's ``[B,H,Nk,D]`` orientation (a copy)."""
        nk = self.shape[3]
        raw = self.value_fp8_transposed.view(torch.uint8)[..., :nk].transpose(-1, -2).contiguous()
        return raw.view(torch.float8_e4m3fn)

    @property
    def value_scale(self) -> torch.Tensor:
        b, h, _nq, _nk, d = self.shape
        return self._view(self.layout.vscale, b * h * d, torch.float32, (b, h, d))

    @property
    def key_mean(self) -> torch.Tensor:
        b, h, _nq, _nk, d = self.shape
        return self._view(self.layout.kmean, b * h * d, torch.float32, (b, h, d))


def workspace_bytes(batch: int, heads: int, nq: int, nk: int, d: int) -> int:
    return int(_native.sage2pp_layout(batch, heads, nq, nk, d).total_bytes)


def prepare_sage_attention_2pp(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    is_causal: bool,
    *,
    workspace: torch.Tensor | None = None,
) -> PreparedSageAttention2pp:
    """Run the quantization prepass into a (new or given) workspace."""
    lib = _native.library()
    b, h, nq, d = query.shape
    nk = key.shape[2]
    layout = _native.sage2pp_layout(b, h, nq, nk, d)
    if workspace is None:
        workspace = torch.empty(int(layout.total_bytes), dtype=torch.uint8, device=query.device)
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_sage2pp_prepass(
                query.data_ptr(), _native.strides3(query), key.data_ptr(), _native.strides3(key),
                value.data_ptr(), _native.strides3(value), _DTYPE_CODES[query.dtype],
                b, h, nq, nk, d, workspace.data_ptr(), workspace.numel(), _stream(query.device),
            ),
            "piper_b200_sage2pp_prepass",
        )
    return PreparedSageAttention2pp(workspace, layout, (b, h, nq, nk, d), query.dtype, is_causal)


def launch_sage_attention_2pp(
    prepared: PreparedSageAttention2pp,
    scale: float,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Run only the fused attention kernel on a prepared workspace."""
    lib = _native.library()
    b, h, nq, nk, d = prepared.shape
    device = prepared.workspace.device
    if out is None:
        out = torch.empty((b, h, nq, d), dtype=prepared.dtype, device=device)
    with torch.cuda.device(device):
        _native.check(
            lib.piper_b200_sage2pp_attention_prepared(
                out.data_ptr(), _DTYPE_CODES[prepared.dtype], b, h, nq, nk, d, float(scale),
                1 if prepared.is_causal else 0, prepared.workspace.data_ptr(), prepared.workspace.numel(),
                _stream(device),
            ),
            "piper_b200_sage2pp_attention_prepared",
        )
    return out


def run_sage_attention_2pp(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: float,
    is_causal: bool,
) -> torch.Tensor:
    """Prepass + fused kernel in one C-ABI call (reference: _run_sage_attention_2pp)."""
    lib = _native.library()
    b, h, nq, d = query.shape
    nk = key.shape[2]
    workspace = torch.empty(workspace_bytes(b, h, nq, nk, d), dtype=torch.uint8, device=query.device)
    out = torch.empty((b, h, nq, d), dtype=query.dtype, device=query.device)
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_sage2pp_fwd(
                query.data_ptr(), _native.strides3(query), key.data_ptr(), _native.strides3(key),
                value.data_ptr(), _native.strides3(value), out.data_ptr(), _DTYPE_CODES[query.dtype],
                b, h, nq, nk, d, float(scale), 1 if is_causal else 0,
                workspace.data_ptr(), workspace.numel(), _stream(query.device),
            ),
            "piper_b200_sage2pp_fwd",
        )
    return out


@torch.library.custom_op("piper_kernels::sage_attention_2pp", mutates_args=())
def b200_sage_attention_2pp(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: float,
    is_causal: bool,
) -> torch.Tensor:
    """Run the prepass and the fused SageAttention2++ kernel on sm_100a."""
    return run_sage_attention_2pp(query, key, value, scale, is_causal)


@b200_sage_attention_2pp.register_fake
def _b200_sage_attention_2pp_fake(
    query: torch.Tensor,
    _key: torch.Tensor,
    _value: torch.Tensor,
    _scale: float,
    _is_causal: bool,
) -> torch.Tensor:
    return torch.empty_like(query, memory_format=torch.contiguous_format)
