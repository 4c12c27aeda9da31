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
    close_fused_allreduce()
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


class TpComm:
    """Peer-memory buffers of the TP group for the fused combine + all-reduce
    (``msv_moe_forward_tp``).  Every rank allocates one shared buffer (receive and result
    areas of flagged words) and one epoch buffer, exports the shared buffer by CUDA IPC, and
    maps every other rank's (handles exchanged over the CPU group).  Collective: all ranks
    construct and close it together.  Whether the mapping worked is agreed over the group: if
    it failed on any rank, every rank unmaps what it mapped and raises the same RuntimeError.
    After a call reports MSV_ERR_TIMEOUT the group is out of step: close it and build a new
    one (zero-filled) on every rank."""

    def __init__(self, max_tokens: int, hidden: int, device: torch.device | None = None, lib=None):
        import ctypes

        from . import _lib
        lib = lib if lib is not None else _lib.load()
        self.lib = lib
        self.world, self.rank = get_tp_size(), get_tp_rank()
        if self.world > _lib.MAX_TP:
            raise ValueError(f"the fused all-reduce supports at most {_lib.MAX_TP} ranks")
        if hidden % (8 * self.world):
            raise ValueError("hidden must be a multiple of 8 * world")
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.max_tokens, self.hidden = max_tokens, hidden
        self.buf = torch.zeros(lib.msv_tp_shared_bytes(max_tokens, hidden), dtype=torch.uint8, device=dev)
        self.epoch = torch.zeros(lib.msv_tp_epoch_bytes() // 4, dtype=torch.int32, device=dev)
        hb = lib.msv_ipc_handle_bytes()
        handle = (ctypes.c_char * hb)()
        off = ctypes.c_uint64(0)
        mine = None
        if lib.msv_ipc_export(self.buf.data_ptr(), handle, ctypes.byref(off)) == _lib.MSV_OK:
            mine = (bytes(handle), int(off.value))
        allh = [mine]
        if self.world > 1:
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=_CPU_GROUP)
        self.imported = []
        ptrs = []
        failed = [p for p, h in enumerate(allh) if h is None]
        for p, h in enumerate(allh):
            if failed:
                break
            if p == self.rank:
                ptrs.append(self.buf.data_ptr())
                continue
            out = ctypes.c_void_p()
            hbuf = (ctypes.c_char * hb).from_buffer_copy(h[0])
            if lib.msv_ipc_import(hbuf, ctypes.c_uint64(h[1]), ctypes.byref(out)) != _lib.MSV_OK:
                failed.append(p)
                break
            self.imported.append(out.value)
            ptrs.append(out.value)
        # every rank learns whether any rank failed
        if not _agree(not failed):
            self._unmap()
            raise RuntimeError("fused all-reduce: CUDA IPC mapping of the peers' buffers failed on a rank"
                               + (f" (this rank: peers {failed})" if failed else ""))
        shared = (ctypes.c_void_p * _lib.MAX_TP)(*(ptrs + [None] * (_lib.MAX_TP - len(ptrs))))
        self.struct = _lib.TpComm(world=self.world, rank=self.rank, max_tokens=max_tokens, hidden=hidden,
                                  shared=shared, epoch=self.epoch.data_ptr())
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        barrier()  # every rank's flags are zero before any rank's first call

    def _unmap(self) -> None:
        for p in self.imported:
            self.lib.msv_ipc_close(p)
        self.imported = []

    def close(self) -> None:
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)
        barrier()  # no rank still reads or writes another's buffer
        self._unmap()


def _agree(ok: bool) -> bool:
    """True on every rank when ``ok`` is true on every rank (over the CPU group)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return ok
    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=_CPU_GROUP)
    return bool(t.item())


_FUSED: TpComm | None = None


def init_fused_allreduce(max_tokens: int, hidden: int, required: bool = True) -> TpComm | None:
    """Enable the fused combine + all-reduce for layers of up to ``max_tokens`` tokens of width
    ``hidden`` (collective).  ``model.qwen35_layer_v2.moe_forward`` then skips ``all_reduce``.
    With ``required=False`` a group whose peer buffers cannot be mapped keeps NCCL's
    all-reduce (every rank alike) and None is returned."""
    global _FUSED
    close_fused_allreduce()
    try:
        _FUSED = TpComm(max_tokens, hidden)
    except RuntimeError:
        if required:
            raise
        _FUSED = None
    return _FUSED


def fused_allreduce_comm(tokens: int, hidden: int) -> TpComm | None:
    """The group's fused all-reduce buffers when they fit a [tokens, hidden] layer, else None."""
    c = _FUSED
    if c is None or get_tp_size() <= 1 or tokens > c.max_tokens or hidden != c.hidden:
        return None
    return c


def close_fused_allreduce() -> None:
    global _FUSED
    if _FUSED is not None:
        _FUSED.close()
        _FUSED = None
