"""Benchmark of the piper_attention forward on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload c4|c2|c3|c5]

One step = one full ``piper_attention`` call (quantization prepass + fused
attention) over one batch of seeded synthetic inputs already resident in HBM.
The default workload is BASELINE configs[3] (c4): B1 H40 N16384 D128 bf16
non-causal, V with a per-feature bias ~N(0,1).  Under torchrun every rank runs
its own shard of B*H (weak scaling: 40 heads per rank, independent data, no
collective on the data path); the reported time is the max over ranks.

``--workload c5`` (B1 H24 N131072) splits the sequence
over the ranks instead (strong scaling): one step is a whole
``ring_piper_attention`` call, with the quantized K/V packs passed around an NCCL
ring and the fp64 column totals all-reduced.

Metric: TOPS = 4*B*H*Nq*Nk*D / t (the reference's formula,
benchmarks/benchmark_attention.py:184-193), summed over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO / "piper-kernels_b200", REPO):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOADS = {
    # name: (B, H, N, D, dtype, causal, description)
    "c4": (1, 40, 16384, 128, torch.bfloat16, False,
           "piper_attention non-causal B1 H40 N16384 D128 bf16 (BASELINE configs[3]); V bias ~N(0,1)"),
    "c2": (2, 24, 4096, 128, torch.bfloat16, False,
           "piper_attention non-causal B2 H24 N4096 D128 bf16 (BASELINE configs[1]); 4 K outlier channels +8, V bias ~N(0,2)"),
    "c3": (4, 32, 8192, 128, torch.float16, True,
           "piper_attention causal B4 H32 N8192 D128 fp16 (BASELINE configs[2]); K offset ~N(0,2)"),
    "c5": (1, 24, 131072, 128, torch.bfloat16, False,
           "piper_attention non-causal sequence-sharded ring B1 H24 N131072 D128 bf16 (BASELINE configs[4]); "
           "V bias ~N(0,1)"),
    "c5causal": (1, 24, 131072, 128, torch.bfloat16, True,
                 "piper_attention CAUSAL sequence-sharded ring, zig-zag shards, B1 H24 N131072 D128 bf16 "
                 "(the c5 shape with the causal mask; not a BASELINE config)"),
}
# Workloads whose sequence is split over the ranks (strong scaling, NCCL ring).
RING_WORKLOADS = {"c5", "c5causal"}
METRIC = "piper_attention TOPS (4*B*H*N^2*D/t) at D=128"
INT8_NOMINAL_TOPS = 4500.0


def make_inputs(name: str, rank: int, device: torch.device):
    """Seeded synthetic Q/K/V with the BASELINE distributions (one rank's shard)."""
    b, h, n, d, dtype, causal, _ = WORKLOADS[name]
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    shape = (b, h, n, d)
    q = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    k = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if name == "c2":
        channels = torch.randperm(d, generator=g, device=device)[:4]
        k[..., channels] += 8.0
        v += torch.randn((b, h, 1, d), generator=g, device=device) * 2.0
    elif name == "c3":
        k += torch.randn((b, h, 1, d), generator=g, device=device) * 2.0
    else:
        v += torch.randn((b, h, 1, d), generator=g, device=device)
    return q.to(dtype), k.to(dtype), v.to(dtype), causal


def make_ring_inputs(name: str, rank: int, world: int, device: torch.device, heads: int | None = None):
    """This rank's rows of the seeded full sequence (identical on every rank).

    The union over ranks is the same tensor for every world size, so the
    ring's output rows equal one GPU's (strong scaling).  Causal workloads use
    the zig-zag layout (chunks r and 2*world-1-r), the others contiguous rows.
    """
    from piper_kernels.attention.piper_attention.ring import zigzag_shard

    b, h, n, d, dtype, causal, _ = WORKLOADS[name]
    h = h if heads is None else heads
    g = torch.Generator(device=device).manual_seed(1000)
    shard = n // world

    def mine(t):
        if causal:
            return zigzag_shard(t, rank, world)
        return t[:, :, rank * shard : (rank + 1) * shard]

    shape = (b, h, n, d)
    q = mine(torch.randn(shape, generator=g, device=device)).to(dtype).contiguous()
    k = mine(torch.randn(shape, generator=g, device=device)).to(dtype).contiguous()
    v = mine(torch.randn(shape, generator=g, device=device))
    v = (v + torch.randn((b, h, 1, d), generator=g, device=device)).to(dtype).contiguous()
    return q, k, v


def attention_ops(b: int, h: int, nq: int, nk: int, d: int) -> float:
    return 4.0 * b * h * nq * nk * d


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int) -> None:
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks rather than fail
            self._nvml = None
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM))
                self.reasons |= self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self._nvml is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._nvml is not None:
            self._thread.join()

    def summary(self) -> dict:
        reasons = sorted(name for bit, name in self.REASONS.items() if self.reasons & bit and name != "gpu_idle")
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
        }


def profiled_traffic(workload: str):
    """DRAM bytes per attention launch from a committed ncu summary, if present."""
    path = REPO / "profiles" / f"attention_{workload}_traffic.json"
    if path.exists():
        return json.loads(path.read_text()).get("traffic_bytes_per_launch")
    return None


def cpu_baseline(workload: str, steps: int = 1) -> dict:
    """The oracle (a C port of the reference's portable path) on one head of the workload.

    Heads are independent in the reference, so the sample is one (b,h) slice
    of the seeded inputs at the full sequence length; TOPS scale linearly.
    """
    from oracle import oracle

    b, h, n, d, dtype, causal, _ = WORKLOADS[workload]
    cores = os.cpu_count() or 1
    oracle.build()
    oracle.set_threads(cores)
    if workload in RING_WORKLOADS:
        q, k, v = make_ring_inputs(workload, 0, 1, torch.device("cpu"), heads=1)
    else:
        q, k, v, _ = make_inputs(workload, 0, torch.device("cpu"))
        q, k, v = q[:1, :1], k[:1, :1], v[:1, :1]
    # At N=131072 one head is still ~70 s of CPU work: time the first
    # `rows` queries against the whole sequence (queries are independent, so
    # TOPS scale with the rows; the prepass of all keys is included).
    rows = n if n <= 16384 else 8192
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        prepared = oracle.prepare(q, k, v, causal)
        if rows < n:
            prepared.query_int8 = np.ascontiguousarray(prepared.query_int8[:, :, :rows])
            prepared.query_scale = np.ascontiguousarray(prepared.query_scale[:, :, : rows // 32])
        oracle.attention_prepared(prepared, d**-0.5, causal)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    ops = attention_ops(1, 1, rows, n, d)
    what = "full sequence" if rows == n else f"first {rows} query rows x all {n} keys"
    return {
        "value": ops / t / 1e12,
        "unit": "TOPS",
        "cores": cores,
        "kind": "port",
        "sample": f"1 of {b * h} heads (B1 H1 N{n} D{d}), {what}; {len(times)} run(s), median {t:.2f} s",
        "seconds_per_sample": t * (n / rows),
    }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    b, h, n, d, dtype, causal, desc = WORKLOADS[args.workload]
    base = cpu_baseline(args.workload, steps=max(1, min(args.steps, 2)))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    ring = args.workload in RING_WORKLOADS
    units = b * h * (1 if ring else world)  # ring: the whole sequence is the job
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": base["value"],
        "unit": "TOPS",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": base["seconds_per_sample"] * units * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if ring else "weak",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded randn with the BASELINE distributions)",
        "config": {"workload": desc, "global_batch": b if ring else b * world, "heads": h, "seq_len": n,
                   "head_dim": d},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    import torch.distributed as dist

    from piper_kernels import _native, piper_attention
    from piper_kernels.attention.piper_attention.b200 import (
        launch_piper_attention,
        prepare_piper_attention,
        run_piper_attention_host,
    )

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    b, h, n, d, dtype, causal, desc = WORKLOADS[args.workload]
    q, k, v, causal = make_inputs(args.workload, rank, dev)
    scale = d**-0.5
    ops_rank = attention_ops(b, h, n, n, d) * (0.5 * (n + 1) / n if causal else 1.0)
    ops_full = attention_ops(b, h, n, n, d)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    ws_bytes = int(_native.workspace_layout(b, h, n, n, d).total_bytes)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty_like(q)

    def step(events=None):
        if events is not None:
            events[0].record(stream)
        prepared = prepare_piper_attention(q, k, v, causal, workspace=workspace)
        if events is not None:
            events[1].record(stream)
        launch_piper_attention(prepared, scale, out=out)
        if events is not None:
            events[2].record(stream)

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        barrier()
        if _native.device_status(local) != 0:
            raise RuntimeError("a kernel reported a timed-out wait during warm-up")
        per_step = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        barrier()
        with ClockSampler(local) as clocks:
            start.record(stream)
            for i in range(args.steps):
                step(per_step[i])
            stop.record(stream)
            torch.cuda.synchronize(dev)
        elapsed_ms = max_over_ranks(start.elapsed_time(stop))
        prepass_ms = [e[0].elapsed_time(e[1]) for e in per_step]
        attn_ms = [e[1].elapsed_time(e[2]) for e in per_step]
        attn_avg_ms = max_over_ranks(sum(attn_ms) / len(attn_ms))
        prepass_avg_ms = max_over_ranks(sum(prepass_ms) / len(prepass_ms))
        status = _native.device_status(local)
        if status != 0:
            raise RuntimeError(f"a kernel reported a timed-out wait (status {status:#x})")

        # End to end with host buffers: pinned Q/K/V in, pinned output out,
        # through the library's host-to-host entry point (chunks of heads
        # stream through the GPU with the copies overlapping the kernels).
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        e2e_steps = max(2, min(args.steps, 5))

        def e2e_step():
            run_piper_attention_host(hq, hk, hv, is_causal=causal, out=hout, synchronize=False)

        e2e_step()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
        ref_out = out.cpu().float()
        if ((hout.float() - ref_out).abs() > 1e-3 + ref_out.abs() / 64).any():
            raise RuntimeError("host-to-host output differs from the device-memory operator")

        # The same through the device-memory operator with the copies in
        # series (what a caller gets by moving tensors first).
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

        def serial_step():
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            o = piper_attention(dq, dk, dv, is_causal=causal)
            hout.copy_(o, non_blocking=True)

        serial_step()
        barrier()
        e0.record(stream)
        for _ in range(e2e_steps):
            serial_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        serial_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps

    ms_per_step = elapsed_ms / args.steps
    value = ops_full * world / (ms_per_step * 1e-3) / 1e12
    measured = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) if (REPO / "MEASURED_PEAKS.json").exists() else {}
    bf16_peak = measured.get("bf16_tflops")
    int8_peak = 2.0 * bf16_peak if bf16_peak else 2.0 * 1590.0
    peak_note = "2 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json)" if bf16_peak else "2 x fallback 1.59 PF bf16"
    attn_tops = ops_rank / (attn_avg_ms * 1e-3) / 1e12
    hbm = measured.get("hbm_gbs") or 6650.0
    # Read Q, K, V once (2 B each); write INT8 Q and K codes and the fp16 V codes
    # (1 + 1 + 2 B); plus the scales and per-key vectors.
    prepass_bytes = b * h * n * d * (3 * 2 + 4) + b * h * (n // 32 + n // 64 + 3 * n) * 4
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8",
            "data": "synthetic (seeded randn with the BASELINE distributions; inputs resident in HBM)",
            "config": {
                "workload": desc,
                "global_batch": b * world,
                "heads": h,
                "seq_len": n,
                "head_dim": d,
                "causal": causal,
                "parallelism": f"heads sharded x{world}, no data-path collective",
                "l2": "inputs larger than L2 (Q/K/V of one step = %.0f MB)" % (3 * b * h * n * d * 2 / 1e6),
            },
            "roofline": {
                "bound": "tensor",
                "achieved": attn_tops,
                "peak": int8_peak,
                "unit": "TOP/s",
                "frac": attn_tops / int8_peak,
                "frac_of_nominal_4500": attn_tops / INT8_NOMINAL_TOPS,
                "peak_source": peak_note,
                "kernel": "piper_attention_kernel",
                "ms_per_launch": attn_avg_ms,
                "ops_per_launch": ops_rank,
                "traffic": profiled_traffic(args.workload),
            },
            "prepass": {
                "ms_per_call": prepass_avg_ms,
                "algorithmic_bytes": prepass_bytes,
                "achieved_gbs": prepass_bytes / (prepass_avg_ms * 1e-3) / 1e9,
                "peak_gbs": hbm,
                "frac": prepass_bytes / (prepass_avg_ms * 1e-3) / 1e9 / hbm,
            },
            "kernel_only_tops": ops_full * world / (attn_avg_ms * 1e-3) / 1e12,
            "e2e": {
                "value": ops_full * world / (e2e_ms * 1e-3) / 1e12,
                "unit": "TOPS",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "api": "piper_b200_attention_fwd_host (pinned host buffers, copies overlapped with kernels)",
                "serial_copies_tops": ops_full * world / (serial_ms * 1e-3) / 1e12,
            },
            "gpu_launches": 3 * args.steps,
            "clocks": clocks.summary(),
        }
        if not args.skip_cpu_baseline:
            line["cpu_baseline"] = {kk: vv for kk, vv in cpu_baseline(args.workload).items() if kk != "seconds_per_sample"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_ring(args) -> None:
    """Sequence-sharded workload: every rank holds N/world rows; one step is a
    whole ``ring_piper_attention`` call (column sums, their all-reduce, the
    shard prepass and world attention launches with the K/V ring)."""
    import datetime

    import torch.distributed as dist

    from piper_kernels import _native
    from piper_kernels.attention.piper_attention import b200, ring_piper_attention
    from piper_kernels.attention.piper_attention.ring import _plan

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # High-priority NCCL streams: the ring's send/recv CTAs are scheduled
        # at the next CTA boundary of the attention grid instead of its tail.
        options = dist.ProcessGroupNCCL.Options()
        options.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev, pg_options=options)
    b, h, n, d, dtype, causal, desc = WORKLOADS[args.workload]
    layout = "zigzag" if causal else "contiguous"
    if n % ((128 if causal else 64) * world):
        raise SystemExit(f"N={n} does not split into {world} shards of whole 64-row groups")
    shard = n // world
    q, k, v = make_ring_inputs(args.workload, rank, world, dev)
    scale = d**-0.5
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        for _ in range(args.warmup):
            ring_piper_attention(q, k, v, is_causal=causal, layout=layout)
        barrier()
        if _native.device_status(local) != 0:
            raise RuntimeError("a kernel reported a timed-out wait during warm-up")
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        barrier()
        with ClockSampler(local) as clocks:
            start.record(stream)
            for _ in range(args.steps):
                ring_piper_attention(q, k, v, is_causal=causal, layout=layout)
            stop.record(stream)
            torch.cuda.synchronize(dev)
        elapsed_ms = max_over_ranks(start.elapsed_time(stop))

        # The dominant kernel alone: one middle ring step's launch (state in and
        # out) over a resident K/V pack of this rank's shard shape.  For the
        # zig-zag layout that is one fully visible (query chunk, key chunk) pair.
        prepared = b200.shard_column_sums(q, k, v, causal)
        b200.shard_prepass(q, k, v, prepared, total_keys=n)
        state = torch.empty(b200.state_bytes(b, h, shard, d) // 4, dtype=torch.float32, device=dev)
        mode = _native.STATE_LOAD | _native.STATE_STORE
        if causal:
            launch_rows = shard // 2
            span = dict(query_range=(launch_rows, launch_rows), key_range=(0, launch_rows), causal_shift=n)
        else:
            launch_rows = shard
            span = {}
        b200.attention_shard(prepared, prepared.kv_pack, scale, state=state, state_mode=_native.STATE_STORE, **span)
        for _ in range(2):
            b200.attention_shard(prepared, prepared.kv_pack, scale, state=state, state_mode=mode, **span)
        k0 = torch.cuda.Event(enable_timing=True)
        k1 = torch.cuda.Event(enable_timing=True)
        launches = max(3, min(args.steps, 10))
        k0.record(stream)
        for _ in range(launches):
            b200.attention_shard(prepared, prepared.kv_pack, scale, state=state, state_mode=mode, **span)
        k1.record(stream)
        torch.cuda.synchronize(dev)
        attn_ms = max_over_ranks(k0.elapsed_time(k1) / launches)
        del prepared, state

        # End to end with host buffers: this rank's pinned Q/K/V rows in, its
        # output rows out, the ring in between.
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hout = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        e2e_steps = max(2, min(args.steps, 3))

        def e2e_step():
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            o = ring_piper_attention(dq, dk, dv, is_causal=causal, layout=layout)
            hout.copy_(o, non_blocking=True)

        e2e_step()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
        status = _native.device_status(local)
        if status != 0:
            raise RuntimeError(f"a kernel reported a timed-out wait (status {status:#x})")

    ms_per_step = elapsed_ms / args.steps
    ops_full = attention_ops(b, h, n, n, d)  # the reference's formula (full N^2 even when causal)
    ops_visible = ops_full * ((n + 1) / (2 * n) if causal else 1.0)
    value = ops_full / (ms_per_step * 1e-3) / 1e12
    measured = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) if (REPO / "MEASURED_PEAKS.json").exists() else {}
    bf16_peak = measured.get("bf16_tflops")
    int8_peak = 2.0 * bf16_peak if bf16_peak else 2.0 * 1590.0
    peak_note = "2 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json)" if bf16_peak else "2 x fallback 1.59 PF bf16"
    ops_launch = attention_ops(b, h, launch_rows, launch_rows, d)
    attn_tops = ops_launch / (attn_ms * 1e-3) / 1e12
    launches_per_step = sum(len(st) for st in _plan(rank, world, shard, causal, layout)) if world > 1 else 1
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int8",
            "data": "synthetic (seeded randn with the BASELINE distributions; inputs resident in HBM)",
            "config": {
                "workload": desc,
                "global_batch": b,
                "heads": h,
                "seq_len": n,
                "head_dim": d,
                "causal": causal,
                "parallelism": (f"sequence ring x{world}: NCCL send/recv of K/V code packs "
                                f"({shard} keys per rank), all-reduce of fp64 [2,B,H,D] column totals"),
                "l2": "inputs larger than L2 (Q/K/V shard of one rank = %.0f MB)" % (3 * b * h * shard * d * 2 / 1e6),
            },
            "roofline": {
                "bound": "tensor",
                "achieved": attn_tops,
                "peak": int8_peak,
                "unit": "TOP/s",
                "frac": attn_tops / int8_peak,
                "frac_of_nominal_4500": attn_tops / INT8_NOMINAL_TOPS,
                "peak_source": peak_note,
                "kernel": "piper_attention_kernel (one ring step: state in and out)",
                "ms_per_launch": attn_ms,
                "ops_per_launch": ops_launch,
                "traffic": None,
            },
            "ring_overhead": {
                "attention_ms_per_step": attn_ms * ops_visible / world / ops_launch,
                "ms_per_step": ms_per_step,
                "frac_outside_attention": 1.0 - attn_ms * ops_visible / world / ops_launch / ms_per_step,
                "layout": layout,
                "visible_tops": ops_visible / (ms_per_step * 1e-3) / 1e12,
            },
            "e2e": {
                "value": ops_full / (e2e_ms * 1e-3) / 1e12,
                "unit": "TOPS",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 3 * q.numel() * q.element_size() * world,
                "d2h_bytes_per_step": q.numel() * q.element_size() * world,
            },
            "gpu_launches": (3 + launches_per_step) * args.steps,
            "clocks": clocks.summary(),
        }
        if not args.skip_cpu_baseline and not causal:
            line["cpu_baseline"] = {kk: vv for kk, vv in cpu_baseline(args.workload).items() if kk != "seconds_per_sample"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    parser.add_argument("--skip-cpu-baseline", action="store_true")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in RING_WORKLOADS:
        run_ring(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
