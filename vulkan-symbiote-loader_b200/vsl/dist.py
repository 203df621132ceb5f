"""Process-group plumbing for tensor-parallel engines (one process per GPU).

NCCL carries the data path inside the engine; this module only moves the 128-byte NCCL
unique id from rank 0 to the other ranks and reduces host-side timings, over a gloo
process group (CPU), so it works the same with or without GPUs.
"""
from __future__ import annotations

import datetime
import os


def env():
    """(world_size, rank, local_rank) from the torchrun environment."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return ws, rank, local


def init(world_size: int, timeout_s: float = 300.0):
    """gloo process group for world_size > 1 (MASTER_ADDR defaults to 127.0.0.1).

    The ranks of one engine group live on one node, so NCCL's bootstrap is pointed at the
    loopback interface unless NCCL_SOCKET_IFNAME is already set (its automatic choice can
    be an address the other local ranks cannot reach); tensor traffic still uses NVLink."""
    if world_size <= 1:
        return None
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def broadcast_bytes(dist, data: bytes | None, n: int, src: int = 0) -> bytes:
    """Rank `src` passes `data` (n bytes); every rank returns the same n bytes."""
    import torch
    if dist is None:
        return data
    buf = torch.zeros(n, dtype=torch.uint8)
    if dist.get_rank() == src:
        if data is None or len(data) != n:
            raise ValueError(f"broadcast_bytes: source needs exactly {n} bytes")
        buf = torch.tensor(list(data), dtype=torch.uint8)
    dist.broadcast(buf, src)
    return bytes(buf.tolist())


def nccl_id(dist, make_id=None) -> bytes | None:
    """NCCL unique id created on rank 0 (by `make_id`, default vsl.nccl_unique_id) and shared."""
    if dist is None:
        return None
    if make_id is None:
        import vsl
        make_id = vsl.nccl_unique_id
    return broadcast_bytes(dist, make_id() if dist.get_rank() == 0 else None, 128)


def max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
