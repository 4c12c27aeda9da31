"""Multi-rank host path on CPU: world_size-2 gloo process groups through
muserve_b200.distributed (the NCCL path's plumbing), with the reference's known-answer
all-reduce test (muserve/scripts/test_allreduce.py:31-43) and the intermediate-sharded layer."""
import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from muserve_b200 import distributed as D
    from muserve_b200 import loader
    from oracle import moe_oracle as orc
    D.init_distributed(backend="gloo", timeout_s=60)
    assert D.get_tp_rank() == rank and D.get_tp_size() == world
    # known answer: every rank fills rank+1, the sum is n(n+1)/2, 100 rounds
    for _ in range(100):
        x = torch.full((4096,), float(rank + 1), dtype=torch.bfloat16)
        D.all_reduce(x)
        assert (x == world * (world + 1) // 2).all()
    # intermediate-sharded layer: per-rank partial, one all-reduce
    w = orc.make_layer_weights(256, 16, 256, 256, seed=3)
    hid = orc.make_hidden(16, 256, 4)
    part = orc.moe_forward(hid, loader.shard_moe_weights(w, world, rank, "inter"), 16, 4).float()
    D.all_reduce(part)
    torch.save(part.to(torch.bfloat16), os.path.join(outdir, f"out{rank}.pt"))
    # fused all-reduce host logic: the IPC handles are exchanged rank-indexed over the CPU
    # group, and moe_forward picks the buffers up only for layers that fit them
    import torch.distributed as dist
    got = [None] * world
    dist.all_gather_object(got, (b"handle-%d" % rank, 256 * rank), group=D._CPU_GROUP)
    assert got == [(b"handle-%d" % p, 256 * p) for p in range(world)]
    assert D.fused_allreduce_comm(16, 256) is None  # not initialised

    class Buffers:  # stands in for a TpComm (which needs GPUs)
        max_tokens, hidden = 32, 256
    D._FUSED = Buffers()
    assert D.fused_allreduce_comm(16, 256) is D._FUSED
    assert D.fused_allreduce_comm(33, 256) is None and D.fused_allreduce_comm(16, 512) is None
    D._FUSED = None
    _tpcomm_agreement(D, rank, world)
    D.barrier()
    D.destroy_distributed()


class _FakeIpcLib:
    """Stands in for the library's IPC calls on the CPU; rank `fail_rank` cannot map a peer."""

    def __init__(self, rank, fail_rank):
        self.rank, self.fail_rank, self.closed = rank, fail_rank, []

    def msv_tp_shared_bytes(self, max_tokens, hidden):
        return max_tokens * hidden * 8

    def msv_tp_epoch_bytes(self):
        return 4096

    def msv_ipc_handle_bytes(self):
        return 64

    def msv_ipc_export(self, ptr, handle, off):
        handle[:7] = b"rank-%02d" % self.rank
        off._obj.value = 16
        return 0

    def msv_ipc_import(self, handle, off, out):
        if self.rank == self.fail_rank:
            return -3
        out._obj.value = 0x1000 * (1 + int(bytes(handle[5:7]))) + off.value
        return 0

    def msv_ipc_close(self, ptr):
        self.closed.append(ptr)
        return 0


def _tpcomm_agreement(D, rank, world):
    """TpComm settles the mapping collectively: when one rank cannot map its peers, every rank
    unmaps and raises; otherwise every rank holds every peer's pointer."""
    fake = _FakeIpcLib(rank, fail_rank=1)
    with pytest.raises(RuntimeError, match="IPC mapping"):
        D.TpComm(8, 256, device=torch.device("cpu"), lib=fake)
    # rank 0 had mapped rank 1's buffer before the group gave up: it was unmapped again
    assert fake.closed == ([0x1000 * 2 + 16] if rank == 0 else [])
    fake = _FakeIpcLib(rank, fail_rank=-1)
    c = D.TpComm(8, 256, device=torch.device("cpu"), lib=fake)
    assert c.struct.world == world and c.struct.rank == rank
    for p in range(world):
        want = c.buf.data_ptr() if p == rank else 0x1000 * (1 + p) + 16
        assert c.struct.shared[p] == want
    c.close()
    assert sorted(fake.closed) == sorted(0x1000 * (1 + p) + 16 for p in range(world) if p != rank)


@pytest.mark.timeout(300)
def test_gloo_two_ranks():
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, outdir)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(240)
        assert p.exitcode == 0
    from conftest import assert_close_bf16
    from oracle import moe_oracle as orc
    o0 = torch.load(os.path.join(outdir, "out0.pt"))
    o1 = torch.load(os.path.join(outdir, "out1.pt"))
    assert torch.equal(o0, o1)
    w = orc.make_layer_weights(256, 16, 256, 256, seed=3)
    ref = orc.moe_forward(orc.make_hidden(16, 256, 4), w, 16, 4)
    assert_close_bf16(o0, ref)
