"""Generate golden fixtures by running the REFERENCE's own ``moe_forward`` on CPU.

The reference (``muserve/model/qwen35_layer_v2.py:561-675``) imports MUSA-only modules.
This script:

1. writes stub modules into a temp dir: an empty ``torch_musa``; empty ``mate``,
   ``mate.gdn_decode``, ``mate.gdn_prefill``; and ``mate.gemm`` whose two FP8 GEMMs are the
   oracle's restatement (``oracle/moe_oracle.py``) wrapped to record their inputs/outputs;
2. patches ``muserve.config`` shape constants before importing the layer module (the layer
   binds them at import, ``qwen35_layer_v2.py:26-30``);
3. runs ``moe_forward`` (TP=1 with ``all_reduce`` patched to a no-op, or TP>1 on gloo ranks
   with the reference's ``all_reduce`` unchanged) on seeded synthetic inputs;
4. saves the intermediates as ``tests/golden/<case>.pt``.

Run from the repo root:  ``python tests/golden/make_golden.py [--ref /path/to/reference]``.
The fixtures are committed; tests never need the reference at run time.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import os
import sys
import tempfile
import textwrap

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import moe_oracle as orc  # noqa: E402

STUB_GEMM = textwrap.dedent('''
    import torch
    from oracle import moe_oracle as _orc
    CALLS = []
    def ragged_m_moe_gemm_8bit(a_pair, w_pair, m_indices, out):
        _orc.ragged_m_moe_gemm_8bit(a_pair, w_pair, m_indices, out)
        CALLS.append(("ragged", a_pair[0].clone(), a_pair[1].clone(), m_indices.clone(), out.clone()))
        return out
    def gemm_fp8_nt_groupwise(a, b, a_scale, b_scale, scale_granularity_mnk=(1, 128, 128),
                              out_dtype=torch.bfloat16):
        o = _orc.gemm_fp8_nt_groupwise(a, b, a_scale, b_scale, scale_granularity_mnk, out_dtype)
        CALLS.append(("dense", a.clone(), a_scale.clone(), None, o.clone()))
        return o
''')


def sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
        t = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def make_stubs() -> str:
    d = tempfile.mkdtemp(prefix="muserve_stubs_")
    os.makedirs(os.path.join(d, "mate"))
    open(os.path.join(d, "torch_musa.py"), "w").close()
    for n in ("__init__.py", "gdn_decode.py", "gdn_prefill.py"):
        open(os.path.join(d, "mate", n), "w").close()
    with open(os.path.join(d, "mate", "gemm.py"), "w") as f:
        f.write(STUB_GEMM)
    return d


def import_reference(ref: str, h: int, e: int, k: int, inter: int, tp: int):
    stubs = make_stubs()
    sys.path[:0] = [stubs, ref, ROOT]
    cfg = importlib.import_module("muserve.config")
    cfg.HIDDEN_SIZE, cfg.NUM_EXPERTS, cfg.NUM_EXPERTS_PER_TOK = h, e, k
    cfg.MOE_INTERMEDIATE, cfg.TP_SIZE = inter, tp
    layer = importlib.import_module("muserve.model.qwen35_layer_v2")
    gemm = importlib.import_module("mate.gemm")
    return layer, gemm


def local_weights(w: dict, tp: int, rank: int) -> dict:
    """Experts ``e % tp == rank`` stacked as ``loader.py:230-264`` does; router and shared
    expert replicated (``loader.py:212-228``)."""
    out = {}
    for key, t in w.items():
        if key.startswith("moe.experts."):
            out[key] = t[rank::tp].contiguous()
        else:
            out[key] = t
    return out


def run_case(ref, name, h, e, k, inter, shared, tokens, wseed, xseed, tp=1, rank=0,
             logits=None, keep_all=False, all_reduce=None):
    layer, gemm = import_reference(ref, h, e, k, inter, tp)
    w = orc.make_layer_weights(h, e, inter, shared, seed=wseed)
    x = orc.make_hidden(tokens, h, xseed)
    wl = local_weights(w, tp, rank)
    if all_reduce is None:
        layer.all_reduce = lambda t: None
    if logits is not None:
        real = layer.bf16_linear

        def fake_linear(xx, ww):
            if ww is wl["moe.gate.weight"]:
                return logits.clone()
            return real(xx, ww)
        layer.bf16_linear = fake_linear
    gemm.CALLS.clear()
    out = layer.moe_forward(x, wl)
    calls = list(gemm.CALLS)
    # the reference's own routing lines, re-run to capture ids/weights (:568-572)
    lg = logits if logits is not None else torch.nn.functional.linear(x, w["moe.gate.weight"]).float()
    scores = torch.softmax(lg, dim=-1)
    tw, tid = torch.topk(scores, k, dim=-1)
    tw = (tw / tw.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
    flat = tid.reshape(-1)
    mask = (flat % tp) == rank
    lid = flat[mask] // tp
    so = lid.argsort(stable=True)
    g = {
        "cfg": dict(hidden=h, experts=e, k=k, inter=inter, shared=shared, tokens=tokens,
                    wseed=wseed, xseed=xseed, tp=tp, rank=rank),
        "hidden_sha": sha(x),
        "logits": lg, "topk_w": tw, "topk_ids": tid,
        "sort_order": so, "inverse_order": so.argsort(), "num_local": int(mask.sum()),
        "output": out,
    }
    ragged = [c for c in calls if c[0] == "ragged"]
    dense = [c for c in calls if c[0] == "dense"]
    g1, g2 = ragged[0], ragged[1]
    g["sorted_expert_ids"] = g1[3]
    g["x_scale"], g["act_scale"] = g1[2], g2[2]
    g["x_fp8_sha"], g["act_fp8_sha"] = sha(g1[1]), sha(g2[1])
    g["gate_up_sha"], g["down_sha"] = sha(g1[4]), sha(g2[4])
    if dense:
        g["shared_down"] = dense[-1][4]
    if keep_all:
        g["x_fp8"], g["act_fp8"] = g1[1], g2[1]
        g["gate_up"], g["down"] = g1[4], g2[4]
    else:
        g["x_fp8_rows"], g["act_fp8_rows"] = g1[1][:4].clone(), g2[1][:4].clone()
        g["gate_up_rows"], g["down_rows"] = g1[4][:4].clone(), g2[4][:4].clone()
    # slices keep their parent storage alive in torch.save: store compact copies only
    return {kk: (v.clone().contiguous() if torch.is_tensor(v) else v) for kk, v in g.items()}


def _tp_worker(rank, world, ref, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = run_case(ref, "c0_tp%d" % world, 2048, 64, 8, 512, 512, 32, 1, 0, tp=world, rank=rank,
                 all_reduce=True)
    torch.save((rank, g["output"], g["sort_order"], g["sorted_expert_ids"], g["num_local"]),
               os.path.join(q, f"rank{rank}.pt"))
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MUSERVE_REF"),
                    help="checkout of the reference (the directory holding muserve/); or set MUSERVE_REF")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    if not a.ref:
        ap.error("the reference checkout is required: --ref PATH or MUSERVE_REF=PATH")
    torch.set_num_threads(os.cpu_count())
    cases = {}
    # H=2048, 64 experts top-8, I=512, shared I=512, 32 tokens, seed 0
    cases["c0"] = lambda: run_case(a.ref, "c0", 2048, 64, 8, 512, 512, 32, 1, 0)
    # tiny case, every intermediate stored in full
    cases["small"] = lambda: run_case(a.ref, "small", 256, 16, 4, 128, 128, 8, 3, 4, keep_all=True)
    # full-shape routing (E=512, top-10, 64 tokens) through the reference's own code path,
    # logits injected: uniform fp32 and bf16-rounded N(0,1.28²)
    gl = torch.Generator().manual_seed(11)
    cases["route_unif"] = lambda: run_case(a.ref, "route_unif", 128, 512, 10, 128, 0, 64, 5, 6,
                                           logits=torch.rand(64, 512, generator=gl))
    gb = torch.Generator().manual_seed(12)
    cases["route_bf16"] = lambda: run_case(
        a.ref, "route_bf16", 128, 512, 10, 128, 0, 64, 5, 6,
        logits=(torch.randn(64, 512, generator=gb) * 1.28).to(torch.bfloat16).float())
    for name, fn in cases.items():
        if a.only and name != a.only:
            continue
        # every case needs a fresh import of the reference (config bound at import)
        for mod in [m for m in sys.modules if m.startswith(("muserve", "mate", "torch_musa"))]:
            del sys.modules[mod]
        g = fn()
        torch.save(g, os.path.join(HERE, f"{name}.pt"))
        print(name, "saved", {kk: tuple(v.shape) for kk, v in g.items() if torch.is_tensor(v)})
    if not a.only or a.only == "c0_tp2":
        import torch.multiprocessing as mp
        ctx = mp.get_context("spawn")
        q = tempfile.mkdtemp(prefix="muserve_tp_")
        ps = [ctx.Process(target=_tp_worker, args=(r, 2, a.ref, 29517, q)) for r in range(2)]
        for p in ps:
            p.start()
        for p in ps:
            p.join()
            assert p.exitcode == 0
        res = [torch.load(os.path.join(q, f"rank{r}.pt")) for r in range(2)]
        assert torch.equal(res[0][1], res[1][1]), "TP ranks disagree after all-reduce"
        torch.save({"cfg": dict(hidden=2048, experts=64, k=8, inter=512, shared=512, tokens=32,
                                wseed=1, xseed=0, tp=2),
                    "output": res[0][1],
                    "sort_order": [r[2] for r in res],
                    "sorted_expert_ids": [r[3] for r in res],
                    "num_local": [r[4] for r in res]}, os.path.join(HERE, "c0_tp2.pt"))
        print("c0_tp2 saved")


if __name__ == "__main__":
    main()
