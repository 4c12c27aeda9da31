"""Tensor-parallel plumbing (``muserve/distributed.py``) over torch.distributed.

GPU tensors go through NCCL (NVLink / NVSwitch on one 8xB200 box); a gloo group carries CPU
tensors and tests.  Unlike the reference (``distributed.py:32``) any world size is accepted.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

_TP_GROUP = None
_CPU_GROUP = None
_TP_RANK = 0
_TP_SIZE = 1


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> None:
    """Initialise the process group from RANK / WORLD_SIZE / LOCAL_RANK (torchrun)."""
    global _TP_GROUP, _CPU_GROUP, _TP_RANK, _TP_SIZE
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kw = dict(backend=backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    _TP_GROUP = dist.group.WORLD
    _TP_RANK, _TP_SIZE = dist.get_rank(), dist.get_world_size()
    _CPU_GROUP = dist.new_group(backend="gloo") if backend != "gloo" else _TP_GROUP


def destroy_distributed() -> None:
    global _TP_GROUP, _CPU_GROUP, _TP_RANK, _TP_SIZE
    if dist.is_initialized():
        dist.destroy_process_group()
    _TP_GROUP, _CPU_GROUP, _TP_RANK, _TP_SIZE = None, None, 0, 1


def get_tp_rank() -> int:
    return dist.get_rank() if dist.is_initialized() else _TP_RANK


def get_tp_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else _TP_SIZE


def get_tp_group():
    return _TP_GROUP if _TP_GROUP is not None else (dist.group.WORLD if dist.is_initialized() else None)


def all_reduce(tensor: torch.Tensor) -> None:
    """In-place SUM all-reduce across the TP group (``muserve/distributed.py:62-64``); a no-op
    when there is no process group or it has one rank."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=get_tp_group())


def all_gather_into_tensor(output: torch.Tensor, input: torch.Tensor) -> None:
    dist.all_gather_into_tensor(output, input, group=get_tp_group())


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier(group=get_tp_group())
