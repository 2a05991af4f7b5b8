"""Benchmark of the piper_attention forward on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload c4|c2|c3|c5|c5causal]

One step = one full ``piper_attention`` call (quantization prepass + fused
attention) over one batch of seeded synthetic inputs already resident in HBM.
The default workload is BASELINE configs[3] (c4): B1 H40 N16384 D128 bf16
non-causal, V with a per-feature bias ~N(0,1).  Every rank generates the same
global problem (``piper_kernels.baseline_configs``); under torchrun rank r
computes only its contiguous slice of the flattened B*H pairs
(``piper_attention_multi_gpu``'s partition; strong scaling of one problem,
no collective on the data path) and the reported time is the max over ranks.

``--workload c5`` (B1 H24 N131072) splits the sequence
over the ranks instead (strong scaling): one step is a whole
``ring_piper_attention`` call, with the quantized K/V packs passed around an NCCL
ring and the fp64 column totals all-reduced.

Metric: TOPS = 4*B*H*Nq*Nk*D / t (the reference's formula,
benchmarks/benchmark_attention.py:184-193) for the whole job.
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

from piper_kernels.baseline_configs import CONFIGS, make_inputs  # noqa: E402

# Workloads whose sequence is split over the ranks (strong scaling, NCCL ring).
RING_WORKLOADS = {"c5", "c5causal"}
BENCH_WORKLOADS = ("c2", "c3", "c4", "c5", "c5causal")
METRIC = "piper_attention TOPS (4*B*H*N^2*D/t) at D=128"
INT8_NOMINAL_TOPS = 4500.0
# Parity bounds of the reference's own GPU tests against its portable path
# (tests/attention/piper_attention/test_triton.py:139-145), plus a cosine floor.
PARITY_MEAN_ABS = 0.003
PARITY_MAX_ABS = 0.12
PARITY_COSINE = 0.9999
# The CPU sample of the c5 workloads: this many query rows of one head
# against all keys (one whole head is about a minute of CPU work).
RING_SAMPLE_ROWS = 2048


def workload(name: str):
    cfg = CONFIGS[name]
    return cfg.batch, cfg.heads, cfg.seq_len, cfg.head_dim, cfg.dtype, cfg.is_causal, cfg.description


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


def oracle_sample(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, rows: int,
                  runs: int = 1) -> dict:
    """The oracle (a C port of the reference's portable path) on one head, timed.

    ``q``/``k``/``v`` are one head, ``[1, 1, N, D]`` on any device: the GPU
    arm's own tensors.  The first ``rows`` query rows attend to all keys
    (query rows are independent, so TOPS scale with them; the prepass of all
    keys is inside the timed region).  Returns the timing, the fp32 output
    rows and the oracle's prepass for parity checks.
    """
    from oracle import oracle

    n, d = k.shape[2], k.shape[3]
    cores = os.cpu_count() or 1
    oracle.build()
    oracle.set_threads(cores)
    qc, kc, vc = (t.detach().cpu() for t in (q, k, v))
    times, out, prepared = [], None, None
    for _ in range(max(1, runs)):
        t0 = time.perf_counter()
        prepared = oracle.prepare(qc[:, :, :rows], kc, vc, causal)
        out = oracle.attention_prepared(prepared, d**-0.5, causal)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    what = "full sequence" if rows == n else f"first {rows} query rows x all {n} keys"
    return {
        "tops": attention_ops(1, 1, rows, n, d) / t / 1e12,  # the metric's formula (full N^2 when causal)
        "seconds": t,
        "runs": len(times),
        "cores": cores,
        "what": what,
        "out": out,
        "prepared": prepared,
    }


def parity_against_oracle(sample: dict, out_gpu: torch.Tensor, prepared_gpu, rows: int) -> dict:
    """GPU output and codes of head 0 against the oracle on the same tensors."""
    ref = torch.from_numpy(sample["out"]).to(out_gpu.dtype).double()
    mine = out_gpu[:, :1, :rows].detach().cpu().double()
    err = (mine - ref).abs()
    cos = torch.nn.functional.cosine_similarity(mine.flatten(), ref.flatten(), dim=0).item()
    p = sample["prepared"]
    n = p.key_int8.shape[2]
    codes = {
        "query_int8": bool(np.array_equal(prepared_gpu.query_int8[:, :1, :rows].cpu().numpy(), p.query_int8)),
        "query_scale": bool(np.array_equal(prepared_gpu.query_scale[:, :1, : (rows + 31) // 32].cpu().numpy(),
                                           p.query_scale)),
        "key_int8": bool(np.array_equal(prepared_gpu.key_int8[:, :1].cpu().numpy(), p.key_int8)),
        "key_scale": bool(np.array_equal(prepared_gpu.key_scale[:, :1].cpu().numpy(), p.key_scale)),
        "value_int8": bool(np.array_equal(prepared_gpu.value_int8[:, :1].cpu().numpy(), p.value_int8)),
        "value_scale": bool(np.array_equal(prepared_gpu.value_scale[:, :1, :n].cpu().numpy(), p.value_scale)),
    }
    result = {
        "sample": f"head (b=0, h=0) of the timed inputs, {sample['what']}; oracle on the same tensors",
        "max_abs": err.max().item(),
        "mean_abs": err.mean().item(),
        "cosine": cos,
        "codes_equal": all(codes.values()),
        "codes": codes,
        "bounds": {"max_abs": PARITY_MAX_ABS, "mean_abs": PARITY_MEAN_ABS, "cosine": PARITY_COSINE},
    }
    result["pass"] = bool(result["codes_equal"] and result["max_abs"] < PARITY_MAX_ABS
                          and result["mean_abs"] < PARITY_MEAN_ABS and cos > PARITY_COSINE)
    return result


def run_reference(args) -> None:
    """The reference arm: the oracle port on the host cores, on the same inputs as the GPU arm.

    One sample = one head of the workload (for c5, its first 2048 query rows
    against all keys), timed whole; ``steps`` counts the samples run and
    ``ms_per_step`` is one sample's time.  The rate scales linearly to the
    whole job (heads and query rows are independent), reported separately.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    b, h, n, d, dtype, causal, desc = workload(args.workload)
    ring = args.workload in RING_WORKLOADS
    gen_device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))) if torch.cuda.is_available() else None
    q, k, v = make_inputs(args.workload, gen_device or "cpu")
    q, k, v = (t[:1, :1].cpu() for t in (q, k, v))
    rows = RING_SAMPLE_ROWS if ring else n
    samples = max(1, min(args.steps, 2))
    s = oracle_sample(q, k, v, causal, rows, runs=samples)
    full_ops = attention_ops(b, h, n, n, d)
    sample_ops = attention_ops(1, 1, rows, n, d)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": s["tops"],
        "unit": "TOPS",
        "n_gpus": args.gpus,
        "steps": s["runs"],
        "warmup": 0,
        "requested_steps": args.steps,
        "requested_warmup": args.warmup,
        "ms_per_step": s["seconds"] * 1e3,
        "step": "one sample: " + s["what"] + " of one head",
        "extrapolated_ms_per_job": s["seconds"] * full_ops / sample_ops * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded randn with the BASELINE distributions; the GPU arm's own tensors)"
                if gen_device is not None else "synthetic (seeded randn with the BASELINE distributions)",
        "config": {"workload": desc, "global_batch": b, "heads": h, "seq_len": n, "head_dim": d},
        "cpu_baseline": {
            "value": s["tops"], "unit": "TOPS", "cores": s["cores"], "kind": "port",
            "value_per_core": s["tops"] / s["cores"],
            "sample": f"1 of {b * h} heads (B1 H1 N{n} D{d}), {s['what']}; {s['runs']} run(s), "
                      f"median {s['seconds']:.2f} s",
        },
        "e2e": {"value": s["tops"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _plan_kernels(b: int, h: int, nq: int, nk: int, d: int, causal: bool) -> int:
    """Kernels one prepared attention call launches (the attention kernel, plus the split merge)."""
    from piper_kernels._targets import AcceleratorTarget
    from piper_kernels.attention.piper_attention._policy import select_execution_plan

    target = AcceleratorTarget.from_device(torch.device("cuda", torch.cuda.current_device()))
    return select_execution_plan(target, batch=b, heads=h, query_length=nq, key_length=nk, head_dim=d,
                                 is_causal=causal).kernels


def run_b200(args) -> None:
    import torch.distributed as dist

    from piper_kernels import _native, piper_attention
    from piper_kernels.attention.piper_attention.b200 import (
        launch_piper_attention,
        prepare_piper_attention,
        run_piper_attention_host,
    )
    from piper_kernels.attention.piper_attention.multi_gpu import head_partition, local_heads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    b, h, n, d, dtype, causal, desc = workload(args.workload)
    # The global problem, identical on every rank; this rank keeps its B*H slice.
    q_all, k_all, v_all = make_inputs(args.workload, dev)
    q, k, v = (local_heads(t, rank, world).contiguous() for t in (q_all, k_all, v_all))
    del q_all, k_all, v_all
    units = q.shape[1]
    first_unit = head_partition(b * h, world)[rank][0]
    scale = d**-0.5
    causal_factor = 0.5 * (n + 1) / n if causal else 1.0
    ops_rank = attention_ops(1, units, n, n, d) * causal_factor
    ops_job = attention_ops(b, h, n, n, d)  # the reference's formula (full N^2 even when causal)

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
    ws_bytes = int(_native.workspace_layout(1, units, n, n, d).total_bytes)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty_like(q)
    prepared = None

    def step(events=None):
        nonlocal prepared
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

        # End to end with host buffers: this rank's pinned Q/K/V slice in, its
        # pinned output slice out, through the library's host-to-host entry
        # point (chunks of heads stream through the GPU with the copies
        # overlapping the kernels).
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
    value = ops_job / (ms_per_step * 1e-3) / 1e12
    measured = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) if (REPO / "MEASURED_PEAKS.json").exists() else {}
    bf16_peak = measured.get("bf16_tflops")
    int8_peak = 2.0 * bf16_peak if bf16_peak else 2.0 * 1590.0
    peak_note = "2 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json)" if bf16_peak else "2 x fallback 1.59 PF bf16"
    attn_tops = ops_rank / (attn_avg_ms * 1e-3) / 1e12
    hbm = measured.get("hbm_gbs") or 6650.0
    # Compulsory bytes of the prepass for this rank's slice: read Q, K, V once
    # (2 B each); write INT8 Q and K codes and the V codes (stored as fp16,
    # 2 B); plus the per-group scales and the three per-key vectors.
    elems = units * n * d
    prepass_bytes = elems * (3 * 2 + 1 + 1 + 2) + units * (n // 32 + n // 64 + 3 * n) * 4
    prepass_bytes_int8_v = prepass_bytes - elems  # the same with INT8 V codes (1 B), the survey's count
    launches = (2 + _plan_kernels(1, units, n, n, d, causal)) * args.steps
    if rank == 0:
        parallelism = ("one GPU" if world == 1 else
                       f"B*H split x{world}: rank r runs a contiguous slice of the {b * h} (b,h) pairs "
                       f"({units} on rank 0), no data-path collective")
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
                "parallelism": parallelism,
                "units_rank0": units,
                "l2": "inputs larger than L2 (Q/K/V of one rank's step = %.0f MB)" % (3 * elems * 2 / 1e6),
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
                "traffic": profiled_traffic(args.workload) if world == 1 else None,
            },
            "prepass": {
                "ms_per_call": prepass_avg_ms,
                "algorithmic_bytes": prepass_bytes,
                "achieved_gbs": prepass_bytes / (prepass_avg_ms * 1e-3) / 1e9,
                "peak_gbs": hbm,
                "frac": prepass_bytes / (prepass_avg_ms * 1e-3) / 1e9 / hbm,
                "frac_int8_v_bytes": prepass_bytes_int8_v / (prepass_avg_ms * 1e-3) / 1e9 / hbm,
            },
            "kernel_only_tops": ops_job / (attn_avg_ms * 1e-3) / 1e12,
            "e2e": {
                "value": ops_job / (e2e_ms * 1e-3) / 1e12,
                "unit": "TOPS",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 3 * q.numel() * q.element_size() * world,
                "d2h_bytes_per_step": out.numel() * out.element_size() * world,
                "api": "piper_b200_attention_fwd_host (pinned host buffers, copies overlapped with kernels)",
                "serial_copies_tops": ops_job / (serial_ms * 1e-3) / 1e12,
            },
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if first_unit == 0 and not args.skip_cpu_baseline:
            # Head (0, 0) of the global problem is rank 0's first pair: the
            # oracle runs on those very tensors, timed (the CPU baseline, at
            # one GPU) and compared with the GPU's output and codes (parity).
            sample = oracle_sample(q[:, :1], k[:, :1], v[:, :1], causal, n)
            line["parity"] = parity_against_oracle(sample, out, prepared, n)
            if world == 1:
                line["cpu_baseline"] = {
                    "value": sample["tops"], "unit": "TOPS", "cores": sample["cores"], "kind": "port",
                    "sample": f"head (0,0) of the timed inputs (B1 H1 N{n} D{d}), {sample['what']}; "
                              f"{sample['seconds']:.2f} s",
                }
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
    from piper_kernels.attention.piper_attention.ring import zigzag_shard

    b, h, n, d, dtype, causal, desc = workload(args.workload)
    layout = "zigzag" if causal else "contiguous"
    if n % ((128 if causal else 64) * world):
        raise SystemExit(f"N={n} does not split into {world} shards of whole 64-row groups")
    shard = n // world
    # The global sequence, identical on every rank; this rank keeps its rows
    # (chunks r and 2*world-1-r of 2*world for the zig-zag layout).
    q_all, k_all, v_all = make_inputs(args.workload, dev)
    if causal:
        q, k, v = (zigzag_shard(t, rank, world).contiguous() for t in (q_all, k_all, v_all))
    else:
        q, k, v = (t[:, :, rank * shard : (rank + 1) * shard].contiguous() for t in (q_all, k_all, v_all))
    del q_all, k_all, v_all
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
                out_last = ring_piper_attention(q, k, v, is_causal=causal, layout=layout)
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
        del state
        parity = None
        sample = None
        if world == 1 and not args.skip_cpu_baseline:
            # One GPU holds the whole sequence: the oracle runs on head (0,0)
            # of the timed tensors (its first rows against all keys), timed
            # (the CPU baseline) and compared with the timed output and the
            # prepass codes of the same head (parity).
            sample = oracle_sample(q[:, :1], k[:, :1], v[:, :1], causal, RING_SAMPLE_ROWS)
            parity = parity_against_oracle(sample, out_last, prepared, RING_SAMPLE_ROWS)
        del prepared, out_last

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
        if parity is not None:
            line["parity"] = parity
            line["cpu_baseline"] = {
                "value": sample["tops"], "unit": "TOPS", "cores": sample["cores"], "kind": "port",
                "sample": f"head (0,0) of the timed inputs (B1 H1 N{n} D{d}), {sample['what']}; "
                          f"{sample['seconds']:.2f} s",
            }
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
    parser.add_argument("--workload", choices=BENCH_WORKLOADS, default="c4")
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
