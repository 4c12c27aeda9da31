"""Weighted combine fused with the TP all-reduce over NVLink peer memory
(qwen35_layer_v2.py:657-662 with distributed.py:62-64).

On one GPU a group of one runs the same fused kernel (its flag exchange is with itself) and
must equal the plain combine bit for bit, call after call and inside a CUDA graph.  With two
or more GPUs, child processes (one per GPU) run the intermediate-sharded layer through the
fused path and through NCCL: at two ranks both sum two bf16 partials in fp32 with one
rounding, so the outputs are identical; every rank holds the same bits; and the result matches
the unsharded oracle within the path's tolerance."""
import os
import socket

import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import moe
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def _layer(cuda, h=1024, e=64, inter=512, seed=3):
    w = orc.make_layer_weights(h, e, inter, inter, seed=seed)
    return {k: v.to(cuda) for k, v in w.items() if torch.is_tensor(v)}


def _group_of_one(cuda, max_tokens, hidden):
    """A TpComm of one rank without a process group."""
    import ctypes

    from muserve_b200 import _lib
    lib = _lib.load()

    class One:
        pass
    c = One()
    c.buf = torch.zeros(lib.msv_tp_shared_bytes(max_tokens, hidden), dtype=torch.uint8, device=cuda)
    c.epoch = torch.zeros(lib.msv_tp_epoch_bytes() // 4, dtype=torch.int32, device=cuda)
    shared = (ctypes.c_void_p * _lib.MAX_TP)(c.buf.data_ptr())
    c.struct = _lib.TpComm(world=1, rank=0, max_tokens=max_tokens, hidden=hidden, shared=shared,
                           epoch=c.epoch.data_ptr())
    return c


@pytest.mark.parametrize("T", [1, 37, 300])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_fused_group_of_one_equals_combine(cuda, T, mode):
    w = _layer(cuda)
    x = orc.make_hidden(T, 1024, 5).to(cuda)
    lg = orc.make_hidden(T, 64, 6).float().to(cuda)
    comm = _group_of_one(cuda, 512, 1024)
    ref = moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, combine_mode=mode)
    for _ in range(3):  # the epochs advance call after call
        got = moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, combine_mode=mode, comm=comm)
        assert torch.equal(got, ref)
    moe.check_device_error()


def test_fused_group_of_one_varying_calls(cuda):
    """One group, calls whose token count (above and below the grid cap) and combine mode
    change from call to call: each token keeps its CTA and flag counter, so every call equals
    the plain combine bit for bit.  At H=4096 a CTA has 512 threads and the grid cap is a few
    hundred CTAs, so 300 and 700 tokens wrap around it."""
    w = _layer(cuda, h=4096, e=16, inter=256)
    comm = _group_of_one(cuda, 700, 4096)
    calls = [(300, 0), (4, 1), (37, 2), (300, 0), (700, 2), (300, 1), (1, 0), (700, 0), (300, 0)]
    for i, (T, mode) in enumerate(calls):
        x = orc.make_hidden(T, 4096, 40 + i).to(cuda)
        lg = orc.make_hidden(T, 16, 60 + i).float().to(cuda)
        ref = moe.moe_layer(x, w, top_k=4, num_experts=16, router_logits=lg, combine_mode=mode)
        got = moe.moe_layer(x, w, top_k=4, num_experts=16, router_logits=lg, combine_mode=mode, comm=comm)
        assert torch.equal(got, ref), (T, mode)
    moe.check_device_error()


def test_fused_group_of_one_in_a_graph(cuda):
    w = _layer(cuda)
    x = orc.make_hidden(64, 1024, 7).to(cuda)
    lg = orc.make_hidden(64, 64, 8).float().to(cuda)
    comm = _group_of_one(cuda, 64, 1024)
    ref = moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg)
    out = torch.empty_like(ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, comm=comm, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, comm=comm, out=out)
    for _ in range(4):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    moe.check_device_error()
    g.reset()


def test_fused_rejects_bad_groups(cuda):
    w = _layer(cuda)
    x = orc.make_hidden(70, 1024, 9).to(cuda)
    lg = orc.make_hidden(70, 64, 10).float().to(cuda)
    comm = _group_of_one(cuda, 64, 1024)  # too few rows for 70 tokens
    with pytest.raises(AssertionError):
        moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, comm=comm)


def test_fused_wait_times_out_and_reports(cuda):
    """Failure detection without a fault: a group of two on one GPU whose second rank never
    runs.  Rank 0's kernel pushes its pieces and then waits for rank 1's, which never come;
    after its 2 s limit it ends, the error word reports MSV_ERR_TIMEOUT, and the context stays
    usable (a later plain layer gives the same bits as before)."""
    import ctypes

    from muserve_b200 import _lib
    lib = _lib.load()
    w = _layer(cuda)
    x = orc.make_hidden(4, 1024, 14).to(cuda)
    lg = orc.make_hidden(4, 64, 15).float().to(cuda)
    ref = moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg)
    moe.check_device_error()
    bufs = [torch.zeros(lib.msv_tp_shared_bytes(16, 1024), dtype=torch.uint8, device=cuda) for _ in range(2)]
    epoch = torch.zeros(lib.msv_tp_epoch_bytes() // 4, dtype=torch.int32, device=cuda)

    class Two:
        pass
    comm = Two()
    comm.struct = _lib.TpComm(world=2, rank=0, max_tokens=16, hidden=1024,
                              shared=(ctypes.c_void_p * _lib.MAX_TP)(bufs[0].data_ptr(), bufs[1].data_ptr()),
                              epoch=epoch.data_ptr())
    moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg, comm=comm)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="status -4"):
        moe.check_device_error()
    moe.check_device_error()  # the check clears the error word
    again = moe.moe_layer(x, w, top_k=6, num_experts=64, router_logits=lg)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, T, result_dir):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from muserve_b200 import distributed as D
    from muserve_b200.loader import shard_moe_weights
    from muserve_b200.model import qwen35_layer_v2 as v2
    D.init_distributed(backend="nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    full = orc.make_layer_weights(1024, 64, 512, 512, seed=11)
    x = orc.make_hidden(T, 1024, 12)
    lg = orc.make_hidden(T, 64, 13).float()
    shard = {k: v.to(dev) for k, v in shard_moe_weights(full, world, rank, "inter").items() if torch.is_tensor(v)}
    xd, lgd = x.to(dev), lg.to(dev)
    # NCCL: this rank's partial, then the all-reduce
    nccl = moe.moe_layer(xd, shard, top_k=6, num_experts=64, router_logits=lgd)
    dist.all_reduce(nccl)
    nccl_v2 = v2.moe_forward(xd, shard, top_k=6)
    comm = D.init_fused_allreduce(512, 1024)
    fused = [moe.moe_layer(xd, shard, top_k=6, num_experts=64, router_logits=lgd, comm=comm).clone()
             for _ in range(3)]
    fused_v2 = v2.moe_forward(xd, shard, top_k=6)  # the drop-in path picks the fused buffers up
    torch.cuda.synchronize()
    moe.check_device_error()
    torch.save({"nccl": nccl.cpu(), "fused": [f.cpu() for f in fused], "nccl_v2": nccl_v2.cpu(),
                "fused_v2": fused_v2.cpu()}, os.path.join(result_dir, f"r{rank}.pt"))
    D.destroy_distributed()


@pytest.mark.parametrize("world,T", [(1, 37), (2, 5), (2, 256)])
def test_fused_allreduce_ranks(cuda, tmp_path, world, T):
    """A real process group per GPU through distributed.TpComm (IPC export/import and the
    group's agreement on it); a group of one runs on any box."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    for r in range(world):
        for f in res[r]["fused"]:
            assert torch.equal(f, res[0]["fused"][0])       # every rank, every call: the same bits
        assert torch.equal(res[r]["fused"][0], res[r]["nccl"])  # up to two ranks: equal to NCCL's sum
        assert torch.equal(res[r]["fused_v2"], res[r]["nccl_v2"])
    full = orc.make_layer_weights(1024, 64, 512, 512, seed=11)
    x = orc.make_hidden(T, 1024, 12)
    lg = orc.make_hidden(T, 64, 13).float()
    ref = orc.moe_forward(x, full, 64, 6, logits=lg)
    assert_close_bf16(res[0]["fused"][0].float(), ref.float())


# ── BASELINE config 3 shapes on 2, 4 and 8 GPUs ─────────────────────────────────────────────

C3 = dict(H=4096, E=512, K=10, I=1024, T=256)


def _c3_inputs(dev):
    from muserve_b200 import synthetic
    w = synthetic.make_layer_weights(C3["H"], C3["E"], C3["I"], C3["I"], seed=1, device=dev)
    x = synthetic.make_hidden(C3["T"], C3["H"], seed=2, device=dev)
    lg = synthetic.uniform_logits(C3["T"], C3["E"], seed=3, device=dev)
    return w, x, lg


def _rank_main_c3(rank, world, port, result_dir):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from muserve_b200 import distributed as D
    from muserve_b200.loader import shard_moe_weights
    D.init_distributed(backend="nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    w, x, lg = _c3_inputs(dev)
    shard = {k: v for k, v in shard_moe_weights(w, world, rank, "inter").items() if torch.is_tensor(v)}
    del w
    torch.cuda.empty_cache()
    kw = dict(top_k=C3["K"], num_experts=C3["E"], router_logits=lg)
    partial = moe.moe_layer(x, shard, **kw)
    nccl = partial.clone()
    dist.all_reduce(nccl)
    comm = D.init_fused_allreduce(C3["T"], C3["H"])
    fused = [moe.moe_layer(x, shard, comm=comm, **kw).clone() for _ in range(3)]
    torch.cuda.synchronize()
    moe.check_device_error()
    torch.save({"partial": partial.cpu(), "nccl": nccl.cpu(), "fused": [f.cpu() for f in fused]},
               os.path.join(result_dir, f"r{rank}.pt"))
    D.destroy_distributed()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_c3_ranks(cuda, tmp_path, world):
    """BASELINE config 3 (H=4096, 512 experts top-10 + shared, I/TP = 1024/world, 256 tokens)
    on `world` GPUs, one process per GPU, through the fused combine + all-reduce: every rank
    holds the same bits on every call; the result equals, bit for bit, the rank partials
    summed in rank order in fp32 with one bf16 rounding (the emulated sum that
    test_gpu_tp_c3.py checks against the oracle); each rank's partial equals the one computed
    with its shard on GPU 0; NCCL's all-reduce agrees within the bf16 bar (bit for bit at two
    ranks)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from muserve_b200.loader import shard_moe_weights
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_c3, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    w, x, lg = _c3_inputs(cuda)
    total = torch.zeros(C3["T"], C3["H"], dtype=torch.float32)
    for r in range(world):
        wr = {k: v for k, v in shard_moe_weights(w, world, r, "inter").items() if torch.is_tensor(v)}
        part = moe.moe_layer(x, wr, top_k=C3["K"], num_experts=C3["E"], router_logits=lg).cpu()
        assert torch.equal(part, res[r]["partial"]), f"rank {r} partial differs from the same shard on GPU 0"
        total += part.float()
        del wr
    emulated = total.to(torch.bfloat16)
    for r in range(world):
        for f in res[r]["fused"]:
            assert torch.equal(f, emulated)
        if world == 2:
            assert torch.equal(res[r]["nccl"], emulated)
        assert_close_bf16(res[r]["nccl"].float(), emulated.float())
    full = moe.moe_layer(x, w, top_k=C3["K"], num_experts=C3["E"], router_logits=lg).cpu()
    assert_close_bf16(emulated.float(), full.float())  # unsharded layer: differs by partial rounding only
    del w
    torch.cuda.empty_cache()
