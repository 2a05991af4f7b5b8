"""B200 backend of Piper Attention: custom op over the sm_100a C ABI.

Replaces the reference's Triton backend
(Piper Kernels 0.2.1, ``src/piper_kernels/attention/piper_attention/triton.py``):

* ``torch.ops.piper_kernels.piper_attention(query, key, value, scale, is_causal)``
  is registered with the same name, schema and fake implementation
  (triton.py:984-1010), so ``torch.compile(fullgraph=True)`` traces it as one
  opaque op;
* ``prepare_piper_attention`` / ``launch_piper_attention`` reproduce the
  reference's prepare/launch split (triton.py:772-951) used by benchmarks;
* all device memory (output and one workspace holding every intermediate)
  is allocated here through torch's caching allocator on the query's device,
  and the kernels run on the current torch stream of that device.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import TYPE_CHECKING

import torch

from ... import _native

if TYPE_CHECKING:
    from ._policy import PiperAttentionExecutionPlan

_DTYPE_CODES = {torch.float16: _native.FLOAT16, torch.bfloat16: _native.BFLOAT16}


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass(frozen=True)
class PreparedPiperAttention:
    """Workspace of one call plus typed views of its intermediates.

    The views alias ``workspace``; they match the reference's prepared tensors
    (triton.py:754-769) except that V codes are stored transposed
    ``[B,H,D,Nk_pad]`` as fp16 (the INT8 values exactly; the INT8 views are
    converted copies) and scales are per group (``[B,H,ceil(N/32|64)]``).
    """

    workspace: torch.Tensor
    layout: _native.WorkspaceLayout
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
    def key_int8(self) -> torch.Tensor:
        b, h, _nq, nk, d = self.shape
        return self._view(self.layout.k8, b * h * nk * d, torch.int8, (b, h, nk, d))

    @property
    def value_f16_transposed(self) -> torch.Tensor:
        """``[B,H,D,Nk_pad]`` V codes as stored for the fp16 PV MMA (exact INT8 values)."""
        b, h, _nq, _nk, d = self.shape
        pad = self.layout.nk_pad
        return self._view(self.layout.v8t, b * h * d * pad, torch.float16, (b, h, d, pad))

    @property
    def value_int8_transposed(self) -> torch.Tensor:
        """``[B,H,D,Nk_pad]`` INT8 V codes (a copy of the fp16 store, exactly converted)."""
        return self.value_f16_transposed.to(torch.int8)

    @property
    def value_int8(self) -> torch.Tensor:
        """V codes in the reference's ``[B,H,Nk,D]`` orientation (a copy)."""
        nk = self.shape[3]
        return self.value_int8_transposed[..., :nk].transpose(-1, -2).contiguous()

    @property
    def query_scale(self) -> torch.Tensor:
        b, h = self.shape[:2]
        g = self.layout.q_groups
        return self._view(self.layout.qscale, b * h * g, torch.float32, (b, h, g))

    @property
    def key_scale(self) -> torch.Tensor:
        b, h = self.shape[:2]
        g = self.layout.k_groups
        return self._view(self.layout.kscale, b * h * g, torch.float32, (b, h, g))

    @property
    def value_scale(self) -> torch.Tensor:
        b, h, _nq, nk, _d = self.shape
        pad = self.layout.nk_pad
        return self._view(self.layout.vscale, b * h * pad, torch.float32, (b, h, pad))[..., :nk]

    @property
    def key_mean(self) -> torch.Tensor:
        b, h, _nq, _nk, d = self.shape
        return self._view(self.layout.kmean, b * h * d, torch.float32, (b, h, d))

    @property
    def value_mean(self) -> torch.Tensor:
        b, h, _nq, _nk, d = self.shape
        return self._view(self.layout.vmean, b * h * d, torch.float32, (b, h, d))

    @property
    def kv_pack(self) -> torch.Tensor:
        """The K/V operands of this workspace as one contiguous byte span."""
        off = int(self.layout.kv_pack)
        return self.workspace[off : off + int(self.layout.kv_pack_bytes)]

    @property
    def column_totals(self) -> torch.Tensor:
        """fp64 ``[2,B,H,D]`` K and V column sums written by :func:`shard_column_sums`."""
        b, h, _nq, _nk, d = self.shape
        return self._view(self.layout.totals, 2 * b * h * d, torch.float64, (2, b, h, d))


def workspace_bytes(batch: int, heads: int, nq: int, nk: int, d: int) -> int:
    return int(_native.workspace_layout(batch, heads, nq, nk, d).total_bytes)


def prepare_piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    is_causal: bool,
    *,
    workspace: torch.Tensor | None = None,
) -> PreparedPiperAttention:
    """Run the quantization prepass into a (new or given) workspace."""
    lib = _native.library()
    b, h, nq, d = query.shape
    nk = key.shape[2]
    layout = _native.workspace_layout(b, h, nq, nk, d)
    if workspace is None:
        workspace = torch.empty(int(layout.total_bytes), dtype=torch.uint8, device=query.device)
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_prepass(
                _ptr(query), _native.strides3(query), _ptr(key), _native.strides3(key),
                _ptr(value), _native.strides3(value), _DTYPE_CODES[query.dtype],
                b, h, nq, nk, d, 1 if is_causal else 0,
                _ptr(workspace), workspace.numel(), _stream(query.device),
            ),
            "piper_b200_prepass",
        )
    return PreparedPiperAttention(workspace, layout, (b, h, nq, nk, d), query.dtype, is_causal)


def default_execution_plan(prepared: PreparedPiperAttention) -> "PiperAttentionExecutionPlan":
    """The plan ``launch_piper_attention`` uses for ``prepared`` on its device."""
    from ..._targets import AcceleratorTarget
    from ._policy import select_execution_plan

    b, h, nq, nk, d = prepared.shape
    return select_execution_plan(
        AcceleratorTarget.from_device(prepared.workspace.device), batch=b, heads=h, query_length=nq,
        key_length=nk, head_dim=d, is_causal=prepared.is_causal,
        split_region=prepared.workspace.numel() >= int(prepared.layout.total_bytes),
    )


def launch_piper_attention(
    prepared: PreparedPiperAttention,
    scale: float,
    *,
    out: torch.Tensor | None = None,
    plan: "PiperAttentionExecutionPlan | None" = None,
) -> torch.Tensor:
    """Run only the fused attention kernel on a prepared workspace.

    ``plan`` overrides the production execution plan (the offline tuner's
    candidates); by default the library selects it.
    """
    lib = _native.library()
    b, h, nq, nk, d = prepared.shape
    device = prepared.workspace.device
    if out is None:
        out = torch.empty((b, h, nq, d), dtype=prepared.dtype, device=device)
    with torch.cuda.device(device):
        if plan is None:
            status = lib.piper_b200_attention_prepared(
                _ptr(out), _DTYPE_CODES[prepared.dtype], b, h, nq, nk, d, float(scale),
                1 if prepared.is_causal else 0, _ptr(prepared.workspace), prepared.workspace.numel(),
                _stream(device),
            )
        else:
            native_plan = plan.to_native()
            status = lib.piper_b200_attention_prepared_plan(
                _ptr(out), _DTYPE_CODES[prepared.dtype], b, h, nq, nk, d, float(scale),
                1 if prepared.is_causal else 0, _ptr(prepared.workspace), prepared.workspace.numel(),
                ctypes.byref(native_plan), _stream(device),
            )
        _native.check(status, "piper_b200_attention_prepared")
    return out


def run_piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: float,
    is_causal: bool,
) -> torch.Tensor:
    """Prepass + fused kernel in one C-ABI call (reference: _run_piper_attention)."""
    lib = _native.library()
    b, h, nq, d = query.shape
    nk = key.shape[2]
    layout = _native.workspace_layout(b, h, nq, nk, d)
    workspace = torch.empty(int(layout.total_bytes), dtype=torch.uint8, device=query.device)
    out = torch.empty((b, h, nq, d), dtype=query.dtype, device=query.device)
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_attention_fwd(
                _ptr(query), _native.strides3(query), _ptr(key), _native.strides3(key),
                _ptr(value), _native.strides3(value), _ptr(out), _DTYPE_CODES[query.dtype],
                b, h, nq, nk, d, float(scale), 1 if is_causal else 0,
                _ptr(workspace), workspace.numel(), _stream(query.device),
            ),
            "piper_b200_attention_fwd",
        )
    return out


def host_scratch_bytes(batch: int, heads: int, nq: int, nk: int, d: int) -> int:
    size = ctypes.c_size_t(0)
    _native.check(
        _native.library().piper_b200_host_scratch_bytes(batch, heads, nq, nk, d, ctypes.byref(size)),
        "piper_b200_host_scratch_bytes",
    )
    return int(size.value)


def run_piper_attention_host(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
    is_causal: bool = False,
    out: torch.Tensor | None = None,
    device: torch.device | int | None = None,
    synchronize: bool = True,
) -> torch.Tensor:
    """The forward pass from host tensors to a host tensor (piper_b200_attention_fwd_host).

    ``query``/``key``/``value`` are contiguous CPU tensors (pinned memory lets
    the copies overlap the kernels); the result is written to ``out`` (a
    contiguous CPU tensor, pinned by default).  Heads stream through the GPU
    in chunks, so host-to-device copies, kernels and device-to-host copies
    overlap.  With ``synchronize=False`` the result is complete once the
    device's current stream has finished.
    """
    from .._validation import validate_attention_inputs

    scale = validate_attention_inputs("piper_attention", query, key, value, scale, is_causal)
    for name, t in (("query", query), ("key", key), ("value", value)):
        if t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError(f"run_piper_attention_host {name} must be a contiguous CPU tensor")
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device("cuda", device).index)
    b, h, nq, d = query.shape
    nk = key.shape[2]
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, pin_memory=True)
    elif out.device.type != "cpu" or not out.is_contiguous() or out.shape != query.shape or out.dtype != query.dtype:
        raise ValueError("out must be a contiguous CPU tensor shaped and typed like query")
    with torch.cuda.device(dev):
        scratch = torch.empty(host_scratch_bytes(b, h, nq, nk, d), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        _native.check(
            _native.library().piper_b200_attention_fwd_host(
                _ptr(query), _ptr(key), _ptr(value), _ptr(out), _DTYPE_CODES[query.dtype], b, h, nq, nk, d,
                float(scale), 1 if is_causal else 0, _ptr(scratch), scratch.numel(), stream.cuda_stream,
            ),
            "piper_b200_attention_fwd_host",
        )
        # Freeing `scratch` here is safe: the call made `stream` wait for its
        # last copy, so whatever reuses the memory on `stream` runs after it.
        if synchronize:
            stream.synchronize()
    return out


def shard_column_sums(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    is_causal: bool,
    *,
    workspace: torch.Tensor | None = None,
) -> PreparedPiperAttention:
    """First step of a sequence shard's prepass: its fp64 K/V column totals.

    The totals (``.column_totals``) are to be summed over all shards before
    :func:`shard_prepass`.  ``query`` only fixes the workspace shape.
    """
    lib = _native.library()
    b, h, nq, d = query.shape
    nk = key.shape[2]
    layout = _native.workspace_layout(b, h, nq, nk, d)
    if workspace is None:
        workspace = torch.empty(int(layout.total_bytes), dtype=torch.uint8, device=query.device)
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_shard_column_sums(
                _ptr(key), _native.strides3(key), _ptr(value), _native.strides3(value),
                _DTYPE_CODES[query.dtype], b, h, nq, nk, d, 1 if is_causal else 0,
                _ptr(workspace), workspace.numel(), _stream(query.device),
            ),
            "piper_b200_shard_column_sums",
        )
    return PreparedPiperAttention(workspace, layout, (b, h, nq, nk, d), query.dtype, is_causal)


def shard_prepass(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    prepared: PreparedPiperAttention,
    total_keys: int,
) -> PreparedPiperAttention:
    """Means from the (already summed) column totals, then this shard's codes."""
    lib = _native.library()
    b, h, nq, nk, d = prepared.shape
    with torch.cuda.device(query.device):
        _native.check(
            lib.piper_b200_shard_prepass(
                _ptr(query), _native.strides3(query), _ptr(key), _native.strides3(key),
                _ptr(value), _native.strides3(value), _DTYPE_CODES[query.dtype],
                b, h, nq, nk, d, 1 if prepared.is_causal else 0, int(total_keys),
                _ptr(prepared.workspace), prepared.workspace.numel(), _stream(query.device),
            ),
            "piper_b200_shard_prepass",
        )
    return prepared


def state_bytes(batch: int, heads: int, nq: int, d: int) -> int:
    return int(_native.library().piper_b200_state_bytes(batch, heads, nq, d))


def attention_shard(
    prepared: PreparedPiperAttention,
    kv_pack: torch.Tensor,
    scale: float,
    *,
    key_length: int | None = None,
    state: torch.Tensor | None = None,
    state_mode: int = 0,
    causal_shift: int = 0,
    out: torch.Tensor | None = None,
    query_range: tuple[int, int] | None = None,
    key_range: tuple[int, int] | None = None,
    masked: bool | None = None,
) -> torch.Tensor | None:
    """Attention of this shard's queries over one shard of keys (a K/V pack).

    ``state`` (fp32, :func:`state_bytes` bytes) carries the per-row softmax
    state between key shards; see ``piper_b200_attention_shard``.
    ``query_range`` / ``key_range`` = (begin, count) restrict the launch to
    those query rows and keys (begins multiples of 64); the output and state
    keep their full shapes.  ``masked=False`` runs a causal problem's launch
    without the causal mask, for keys that all precede the queries (the V
    mean of a causal prepass is already zero).  Returns the output unless
    ``state_mode`` stores the state instead.
    """
    lib = _native.library()
    b, h, nq, nk, d = prepared.shape
    nk = nk if key_length is None else int(key_length)
    q0, qn = query_range if query_range is not None else (0, nq)
    k0, kn = key_range if key_range is not None else (0, nk)
    unmasked = masked is False  # an explicit request to drop the causal mask
    causal = prepared.is_causal and not unmasked
    device = prepared.workspace.device
    if out is None and not state_mode & _native.STATE_STORE:
        out = torch.empty((b, h, nq, d), dtype=prepared.dtype, device=device)
    with torch.cuda.device(device):
        _native.check(
            lib.piper_b200_attention_shard_range(
                None if out is None else _ptr(out), _DTYPE_CODES[prepared.dtype], b, h, nq, int(q0), int(qn), nk,
                int(k0), int(kn), d, float(scale), 1 if causal else 0, 0 if unmasked else int(causal_shift),
                _ptr(prepared.workspace), prepared.workspace.numel(), _ptr(kv_pack),
                None if state is None else _ptr(state), int(state_mode), _stream(device),
            ),
            "piper_b200_attention_shard_range",
        )
    return None if state_mode & _native.STATE_STORE else out


@torch.library.custom_op("piper_kernels::piper_attention", mutates_args=())
def b200_piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: float,
    is_causal: bool,
) -> torch.Tensor:
    """Quantization prepass and fused INT8-QK / UINT8xINT8-PV attention on sm_100a."""
    return run_piper_attention(query, key, value, scale, is_causal)


@b200_piper_attention.register_fake
def _b200_piper_attention_fake(
    query: torch.Tensor,
    _key: torch.Tensor,
    _value: torch.Tensor,
    _scale: float,
    _is_causal: bool,
) -> torch.Tensor:
    return torch.empty_like(query, memory_format=torch.contiguous_format)
