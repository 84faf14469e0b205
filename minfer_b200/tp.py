"""Tensor-parallel bring-up for one process per GPU (torchrun).

Every process loads its shard (`Qwen3Model(..., tp_rank=r, tp_size=n)`),
moves it to CUDA, then `connect` exchanges the exchange-region handles over
a torch.distributed group and connects the ranks. Only the handle exchange
uses torch.distributed; the decode-time all-reduces run inside the CUDA
kernels over NVLink peer memory.
"""
from __future__ import annotations

import os


def env_ranks() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process when unset)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' handles, ordered by rank in `group` (torch.distributed)."""
    import torch.distributed as dist

    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    if any(not isinstance(h, (bytes, bytearray)) or len(h) != len(handle) for h in out):
        raise RuntimeError("malformed exchange handle from a peer")
    return [bytes(h) for h in out]


def connect(model, group=None) -> None:
    """Connect a CUDA-resident tensor-parallel model to its peers. The
    torch.distributed rank in `group` must equal the model's tp_rank."""
    import torch.distributed as dist

    if model.info.tp_size == 1:
        return
    if dist.get_world_size(group) != model.info.tp_size or dist.get_rank(group) != model.info.tp_rank:
        raise ValueError("torch.distributed group does not match the model's tp_rank / tp_size")
    model.comm_connect(gather_handles(model.comm_handle(), group))
    dist.barrier(group)
