"""One rank of the NCCL ring check (launched by test_gpu_ring.py under torchrun).

Every rank builds the same full sequence from one seed, runs
``ring_piper_attention`` on its rows over NCCL, and compares them with the
one-GPU operator on the whole sequence, computed on its own GPU, and head 0
with the CPU oracle on the same tensors.  Prints
RING_OK on success; any mismatch raises (non-zero exit).
"""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
for _p in (REPO / "piper-kernels_b200", REPO):
    sys.path.insert(0, str(_p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import oracle  # noqa: E402
from piper_kernels import piper_attention  # noqa: E402
from piper_kernels.attention.piper_attention import ring_piper_attention  # noqa: E402
from piper_kernels.attention.piper_attention.ring import zigzag_shard  # noqa: E402


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    try:
        cases = ((False, torch.bfloat16, 2048, "contiguous"), (True, torch.float16, 1024, "contiguous"),
                 (True, torch.bfloat16, 1024, "zigzag"))
        for is_causal, dtype, n_shard, layout in cases:
            g = torch.Generator(device=dev).manual_seed(123)
            shape = (1, 4, n_shard * world, 128)
            q = torch.randn(shape, generator=g, device=dev).to(dtype)
            k = (torch.randn(shape, generator=g, device=dev) + 1.0).to(dtype)
            v = (torch.randn(shape, generator=g, device=dev) + 0.5).to(dtype)
            if layout == "zigzag":
                def mine_of(t):
                    return zigzag_shard(t, rank, world).contiguous()
            else:
                def mine_of(t):
                    return t[:, :, rank * n_shard : (rank + 1) * n_shard]
            # The last case also waits for every ring step on the host (the
            # failure-detection path), which must not change the result.
            timeout = datetime.timedelta(seconds=30) if layout == "zigzag" else None
            with torch.no_grad():
                mine = ring_piper_attention(mine_of(q), mine_of(k), mine_of(v), is_causal=is_causal, layout=layout,
                                            step_timeout=timeout, abort_on_failure=timeout is not None)
                whole = mine_of(piper_attention(q, k, v, is_causal=is_causal))
            torch.cuda.synchronize()
            err = (mine.float() - whole.float()).abs()
            if not (err.max().item() < 0.02 and err.mean().item() < 2e-4):
                raise AssertionError(f"rank {rank} causal={is_causal} {layout}: max {err.max().item()} "
                                     f"mean {err.mean().item()}")
            # Head 0 against the oracle on the same tensors (the reference's GPU bounds).
            expected = oracle.piper_attention_torch(q[:, :1].cpu(), k[:, :1].cpu(), v[:, :1].cpu(), 128**-0.5,
                                                    is_causal).float()
            ref_err = (mine[:, :1].float().cpu() - mine_of(expected)).abs()
            if not (ref_err.mean().item() < 0.003 and ref_err.max().item() < 0.12):
                raise AssertionError(f"rank {rank} causal={is_causal} {layout} vs oracle: max {ref_err.max().item()}")
        dist.barrier(device_ids=[local])
        print("RING_OK", rank, flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
