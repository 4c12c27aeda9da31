#!/usr/bin/env python
"""MoE-layer benchmark (BASELINE.json metric: MoE-layer tokens/s; HBM GB/s at decode, FP8
TFLOP/s at prefill).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

N = 1  -> BASELINE config 1 (the line's headline): full-shape decode layer (H=4096, 512 experts
          top-10 + shared expert, I=1024) on 64 tokens with uniform random router logits; then
          BASELINE config 2 on the same layer (8192 tokens, routed from the hidden states by the
          library's router GEMM inside every timed step) as the line's "prefill" object.
N > 1  -> BASELINE config 3 (launched by torchrun, one rank per GPU): the same layer at TP=N
          with the expert intermediate sharded (column-parallel gate_up, row-parallel down),
          256 tokens; the per-rank [256,4096] bf16 partials are summed by the combine kernel itself
          over NVLink peer memory (--nccl-allreduce: plain combine + one NCCL all-reduce).  The
          line also carries the same 256-token layer timed unsharded on one GPU
          (same_config_1gpu) and the strong-scaling efficiency against it.
--workload prefill -> BASELINE config 2 alone as the line's headline.
--workload stack   -> BASELINE config 4: the 60-layer MoE decode stack (128 tokens, Zipf(1.2)
          logit prior, RMSNorm + router GEMM + layer per layer) as one CUDA graph at TP=N.

Synthetic seeded data, random-init weights of the full shape.  Timed region: K steps between
barrier + synchronize, CUDA events on the launching stream, max over ranks.  Every step
streams >= 0.8 GB of expert weights per GPU, more than the 126 MB L2, so no flush is needed.
Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "MoE-layer tokens/s"
H, E, K_TOP, INTER, SHARED = 4096, 512, 10, 1024, 1024
STAGES = ["router_topk", "dispatch", "gather_quant", "gemm_gate_up", "gemm_down", "combine"]


def peaks():
    for path in (os.path.join(ROOT, "MEASURED_PEAKS.json"),):
        if os.path.exists(path):
            d = json.load(open(path))
            return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples (SM clock, throttle reasons) during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5:  # sampler running before timing starts
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark(self, on: bool):
        self.active = on
        self.rows.append(["mark", "on" if on else "off"])

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        # samples between the marks (the timed region), else all samples
        rows, inside, sel = self.rows, False, []
        for r in rows:
            if r[0] == "mark":
                inside = r[1] == "on"
                continue
            if inside:
                sel.append(r)
        rows = sel or [r for r in rows if r[0] != "mark"]
        self.rows = rows
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        from muserve_b200 import distributed as D
        D.init_distributed(backend="nccl", timeout_s=120)
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()
    return x


def barrier():
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def expert_bytes(inter: int) -> int:
    w = 3 * H * inter
    s = ((2 * inter // 128) * (H // 128) + (H // 128) * (inter // 128)) * 4
    return w + s


def kernel_bytes(stage: str, n_touched: int, rows: int, inter: int, shared: int, tokens: int) -> int:
    """Algorithmic HBM bytes of one launch: weights + scales of each touched expert (and the
    shared expert) plus the activations the kernel must read and write once."""
    kb_h, kb_i = H // 128, inter // 128
    if stage == "gemm_gate_up":
        w = (n_touched + (1 if shared else 0)) * (2 * inter * H + 2 * kb_i * kb_h * 4)
        return w + rows * (H + kb_h * 4) + rows * (inter + kb_i * 4)
    if stage == "gemm_down":
        w = (n_touched + (1 if shared else 0)) * (H * inter + kb_h * kb_i * 4)
        return w + rows * (inter + kb_i * 4) + rows * H * 2
    raise ValueError(stage)


def kernel_flops(stage: str, rows: int, inter: int) -> int:
    """FP8 MMA FLOPs of one launch: 2 per multiply-add over every (row, output column, k)."""
    if stage == "gemm_gate_up":
        return 2 * rows * (2 * inter) * H
    if stage == "gemm_down":
        return 2 * rows * H * inter
    raise ValueError(stage)


def layer_bytes(n_touched, inter, shared, tokens):
    return (n_touched + (1 if shared else 0)) * expert_bytes(inter) + 2 * tokens * H * 2


def traffic_for(workload: str, kernel: str):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d.get(workload, {}).get(kernel)
    return None


def time_layer(args, lib, dev, w, x, *, tokens, n_exp, logits=None, tp=1, comm=None, want_e2e=True):
    """Time one MoE layer configuration on this GPU the bench's way and return its figures.

    ``logits`` given: the router starts from them (BASELINE configs 1 and 3: uniform random
    logits).  ``logits`` None: every step routes from the hidden states on the library's
    tcgen05 router GEMM (``msv_router_from_hidden``) and then runs the layer on that routing
    (BASELINE config 2 specifies a router gate).  ``tp > 1``: ``w`` is this rank's shard and the
    partials are summed over the group, by the fused combine (``comm``) or by NCCL."""
    import ctypes

    from muserve_b200 import _lib, moe
    from_hidden = logits is None
    inter = w["moe.experts.gate_proj.weight"].shape[1]
    shared = w["moe.shared_expert.gate_proj.weight"].shape[0]
    ws_struct, info = moe.weights_struct(w)
    shape = _lib.MoeShape(tokens=tokens, hidden=H, num_experts=n_exp, top_k=K_TOP, inter=inter, shared_inter=shared,
                          placement=0, tp=1, rank=0, add_shared=1, combine_mode=_lib.COMBINE_V2,
                          weights_dtype=_lib.MSV_BF16)
    nbytes = lib.msv_moe_forward_workspace_size(ctypes.byref(shape))
    wsbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(tokens, H, dtype=torch.bfloat16, device=dev)
    tw = torch.empty(tokens, K_TOP, dtype=torch.bfloat16, device=dev)
    tid = torch.empty(tokens, K_TOP, dtype=torch.int32, device=dev)
    gate_w = w["moe.gate.weight"]
    rbytes = lib.msv_router_workspace_size(tokens, H, n_exp) if from_hidden else 0
    rws = torch.empty(max(rbytes, 256), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    nst = len(STAGES) + 1
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nst + 1)] for _ in range(args.steps)]
    ar_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for row in evs:  # create the event handles before anything is timed
        for e in row:
            e.record(stream)
    # Timed steps record only the two events around the gate_up GEMM, the roofline's kernel
    # (indices 3, 4: each recorded event between kernels costs about 3 us of device time and
    # stops the next launch from overlapping the previous one); the other stages, the down GEMM
    # among them, are timed in separate fully instrumented steps after the timed region.  The
    # extra last event of a row marks the start of the router GEMM when the step routes from
    # the hidden states.
    GEMM_EV = (3, 4)
    ev_arrays = [(ctypes.c_void_p * nst)(*[e.cuda_event if j in GEMM_EV else None for j, e in enumerate(row[:nst])])
                 for row in evs]
    n_prof = min(args.steps, 10)
    evs_p = [[torch.cuda.Event(enable_timing=True) for _ in range(nst + 1)] for _ in range(n_prof)]
    for row in evs_p:
        for e in row:
            e.record(stream)
    ev_arrays_p = [(ctypes.c_void_p * nst)(*[e.cuda_event for e in row[:nst]]) for row in evs_p]
    cref = ctypes.byref(comm.struct) if comm is not None else None
    flags = _lib.FWD_ROUTING_GIVEN if from_hidden else 0
    lg_ptr = None if from_hidden else logits.data_ptr()

    def step(i=None, prof=False):
        if from_hidden:
            if prof:
                evs_p[i][nst].record(stream)
            _lib.check(lib.msv_router_from_hidden(x.data_ptr(), gate_w.data_ptr(), tokens, H, n_exp, K_TOP, 1, 1,
                                                  tw.data_ptr(), _lib.MSV_BF16, tid.data_ptr(), _lib.MSV_I32, None,
                                                  rws.data_ptr(), rws.numel(), sp), "msv_router_from_hidden")
        common = (ctypes.byref(shape), ctypes.byref(ws_struct), x.data_ptr(), lg_ptr, tw.data_ptr(), tid.data_ptr(),
                  out.data_ptr(), flags, wsbuf.data_ptr(), nbytes)
        if i is not None:
            arr = ev_arrays_p[i] if prof else ev_arrays[i]
            if comm is not None:
                rc = lib.msv_moe_forward_tp_profiled(*common, cref, sp, arr)
            else:
                rc = lib.msv_moe_forward_profiled(*common, sp, arr)
        elif comm is not None:
            rc = lib.msv_moe_forward_tp(*common, cref, sp)
        else:
            rc = lib.msv_moe_forward(*common, sp)
        _lib.check(rc, "msv_moe_forward")
        if tp > 1 and comm is None:
            if i is not None and not prof:
                ar_ev[i][0].record(stream)
            dist.all_reduce(out)
            if i is not None and not prof:
                ar_ev[i][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.check(lib.msv_check_device_error(sp), "warmup")
    # routing statistics of the measured step (identical every step)
    counts = torch.bincount(tid.flatten().long(), minlength=n_exp)
    n_touched = int((counts > 0).sum().item())
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    # The clock window: the timed region plus identical untimed steps right before it, enough
    # that the 50 ms nvidia-smi sampler sees the GPU under this load (--clock-window-ms, 500).
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for _ in range(args.warmup):
        step()
    w1.record(stream)
    torch.cuda.synchronize()
    est_ms = max(w0.elapsed_time(w1) / max(args.warmup, 1), 1e-3)
    n_soak = int(max_over_ranks(min(5000, max(0, int(args.clock_window_ms / est_ms) - args.steps))))
    barrier()
    torch.cuda.synchronize()
    with Clocks(torch.cuda.current_device()) as clk:
        clk.mark(True)
        for _ in range(n_soak):
            step()
        t0.record(stream)
        n_launch0 = moe.launch_count()
        for i in range(args.steps):
            step(i)
        n_launches = moe.launch_count() - n_launch0
        t1.record(stream)
        torch.cuda.synchronize()
        clk.mark(False)
    barrier()
    ms_total = max_over_ranks(t0.elapsed_time(t1))
    _lib.check(lib.msv_check_device_error(sp), "timed region")
    # the other stages from fully instrumented steps after the timed region (same collectives on
    # every rank), the gate_up GEMM from the timed steps themselves
    for i in range(n_prof):
        step(i, prof=True)
    torch.cuda.synchronize()
    stage_ms = {s: statistics.mean(evs_p[i][j].elapsed_time(evs_p[i][j + 1]) for i in range(n_prof))
                for j, s in enumerate(STAGES)}
    if from_hidden:  # router GEMM + top-k: from the event before the router to the dispatch
        stage_ms["router_topk"] = statistics.mean(evs_p[i][nst].elapsed_time(evs_p[i][1]) for i in range(n_prof))
    for j, s in enumerate(STAGES):
        if j in GEMM_EV and j + 1 in GEMM_EV:
            stage_ms[s] = statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps))
    ar_ms = statistics.mean(a.elapsed_time(b) for a, b in ar_ev) if (tp > 1 and comm is None) else 0.0
    res = {"ms_total": ms_total, "ms_step": ms_total / args.steps, "value": tokens * args.steps / (ms_total / 1e3),
           "stage_ms": stage_ms, "n_touched": n_touched, "n_launches": n_launches, "ar_ms": ar_ms,
           "inter": inter, "shared": shared,
           "clocks": dict(clk.summary(), window=f"timed region + {n_soak} identical untimed steps just before it")}
    if want_e2e and not args.no_e2e:
        res["e2e"] = time_e2e(args, dev, w, x, logits, tokens=tokens, n_exp=n_exp, tp=tp, comm=comm)
    del wsbuf, rws
    return res


def time_e2e(args, dev, w, x, logits, *, tokens, n_exp, tp, comm):
    """The same metric through the public API from pinned host buffers, every step copying its
    input in and reading its result back.  Pipelined as a serving loop runs it: two buffer sets,
    the input of step i+1 (host -> device stream) and the result of step i-1 (device -> host
    stream) move while step i computes; events keep each buffer from being reused before it is
    read.  The serial form (copy in, compute, copy out, one after the other) is reported beside
    it.  Logits given: ``moe.moe_layer``; from the hidden states: the reference-shaped
    ``model.qwen35_layer_v2.moe_forward`` (router GEMM + layer)."""
    from muserve_b200 import moe as M
    from muserve_b200.model import qwen35_layer_v2 as v2
    from_hidden = logits is None
    hx = x.cpu().pin_memory()
    hl = None if from_hidden else logits.cpu().pin_memory()
    comp = torch.cuda.current_stream(dev)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dxs = [torch.empty_like(x) for _ in range(2)]
    dls = [None if from_hidden else torch.empty_like(logits) for _ in range(2)]
    outs = [torch.empty(tokens, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    hos = [torch.empty(tokens, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    in_ready, in_free, out_ready, out_free = ([torch.cuda.Event() for _ in range(2)] for _ in range(4))
    for b in range(2):
        in_free[b].record(comp)
        out_free[b].record(d2h_s)

    def layer(dx, dl, o):
        if from_hidden:
            o.copy_(v2.moe_forward(dx, w, top_k=K_TOP))
            return
        M.moe_layer(dx, w, top_k=K_TOP, num_experts=n_exp, router_logits=dl, out=o, comm=comm)
        if tp > 1 and comm is None:
            dist.all_reduce(o)

    def piped_step(i):
        b = i & 1
        h2d_s.wait_event(in_free[b])
        with torch.cuda.stream(h2d_s):
            dxs[b].copy_(hx, non_blocking=True)
            if hl is not None:
                dls[b].copy_(hl, non_blocking=True)
        in_ready[b].record(h2d_s)
        comp.wait_event(in_ready[b])
        comp.wait_event(out_free[b])
        layer(dxs[b], dls[b], outs[b])
        in_free[b].record(comp)
        out_ready[b].record(comp)
        d2h_s.wait_event(out_ready[b])
        with torch.cuda.stream(d2h_s):
            hos[b].copy_(outs[b], non_blocking=True)
        out_free[b].record(d2h_s)

    def serial_step(i):
        dxs[0].copy_(hx, non_blocking=True)
        if hl is not None:
            dls[0].copy_(hl, non_blocking=True)
        layer(dxs[0], dls[0], outs[0])
        hos[0].copy_(outs[0], non_blocking=True)

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(comp)
        h2d_s.wait_event(a0)  # no copy starts before the timed region
        for i in range(args.steps):
            fn(i)
        comp.wait_stream(d2h_s)  # the last result is on the host
        a1.record(comp)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a0.elapsed_time(a1))
    ms_e2e = timed(piped_step)
    ms_serial = timed(serial_step)
    return {"value": tokens * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": hx.numel() * 2 + (hl.numel() * 4 if hl is not None else 0),
            "d2h_bytes_per_step": hos[0].numel() * 2, "ms_per_step": ms_e2e / args.steps,
            "api": "model.qwen35_layer_v2.moe_forward (router GEMM + layer)" if from_hidden else "moe.moe_layer",
            "copies": "pipelined: step i+1's input and step i-1's result move while step i computes",
            "serial": {"value": tokens * args.steps / (ms_serial / 1e3), "ms_per_step": ms_serial / args.steps}}


def roofline(r, tokens, *, prefill):
    """Roofline object of the dominant kernel (the longer GEMM) of a time_layer result."""
    hbm, bf16_tf, peak_kind = peaks()
    stage_ms, inter, shared = r["stage_ms"], r["inter"], r["shared"]
    rows = tokens * K_TOP + tokens
    dom = max(("gemm_gate_up", "gemm_down"), key=lambda s: stage_ms[s])
    dom_bytes = kernel_bytes(dom, r["n_touched"], rows, inter, shared, tokens)
    dom_flops = kernel_flops(dom, rows, inter)
    sec = stage_ms[dom] / 1e3
    hbm_part = {"achieved": dom_bytes / sec / 1e9, "peak": hbm, "unit": "GB/s", "peak_kind": peak_kind}
    hbm_part["frac"] = hbm_part["achieved"] / hbm
    if prefill:
        # both bounds (FP8 rate = 2 x the measured bf16 GEMM); the binding one is the longer time:
        # at 160 rows per expert the weights give 320 FLOP/B, under the ~517 FLOP/B ridge, so HBM
        t_hbm, t_tc = dom_bytes / (hbm * 1e9), dom_flops / (2 * bf16_tf * 1e12)
        tensor = {"achieved": dom_flops / sec / 1e12, "peak": 2 * bf16_tf, "unit": "TFLOP/s",
                  "peak_kind": f"2 x {peak_kind} bf16 (e4m3 rate)"}
        tensor["frac"] = tensor["achieved"] / tensor["peak"]
        if t_hbm >= t_tc:
            roof = dict(bound="hbm", kernel=dom, **hbm_part, other={"bound": "tensor", **tensor})
        else:
            roof = dict(bound="tensor", kernel=dom, **tensor, other={"bound": "hbm", **hbm_part})
        roof["algorithmic_flops_per_launch"] = dom_flops
    else:
        roof = dict(bound="hbm", kernel=dom, **hbm_part)
    roof["algorithmic_bytes_per_launch"] = dom_bytes
    return roof, dom


def layer_summary(r, tokens, tp, comm, nccl_allreduce, combine_alone_ms=None):
    """``combine_alone_ms``: the plain combine's stage time of the same batch on one GPU; with the
    fused combine + all-reduce, the all-reduce's own cost is the fused stage minus it."""
    hbm, _, _ = peaks()
    inter, shared, ms_step = r["inter"], r["shared"], r["ms_step"]
    gbs = layer_bytes(r["n_touched"], inter, shared, tokens) / (ms_step / 1e3) / 1e9
    flops = 6 * H * inter * tokens * K_TOP + 6 * H * shared * tokens
    return {"hbm_gbs": gbs, "hbm_frac": gbs / hbm, "n_touched_experts": r["n_touched"],
            "fp8_tflops": flops / (ms_step / 1e3) / 1e12, "stage_ms": r["stage_ms"],
            "allreduce": ("fused into the combine (peer memory)" if comm is not None
                          else ("none" if tp == 1 else ("nccl" if nccl_allreduce else
                                                        "nccl (the peers' buffers could not be mapped)"))),
            "allreduce_ms": r["ar_ms"] if comm is None else None,
            "allreduce_share": (r["ar_ms"] / ms_step if tp > 1 else 0.0) if comm is None else None,
            "combine_allreduce_ms": r["stage_ms"]["combine"] if comm is not None else None,
            "combine_allreduce_share": r["stage_ms"]["combine"] / ms_step if comm is not None else None,
            "allreduce_added_ms": (r["stage_ms"]["combine"] - combine_alone_ms
                                   if comm is not None and combine_alone_ms is not None else None),
            "allreduce_added_share": ((r["stage_ms"]["combine"] - combine_alone_ms) / ms_step
                                      if comm is not None and combine_alone_ms is not None else None),
            "allreduce_added_how": ("fused combine + all-reduce stage minus the plain combine of the same "
                                    "batch on one GPU (same_config_1gpu), over this layer's step"
                                    if comm is not None and combine_alone_ms is not None else None)}


def run_ours(args, world, rank, local):
    from muserve_b200 import _lib, synthetic
    from muserve_b200.loader import shard_moe_weights
    lib = _lib.load()
    dev = torch.device("cuda", local)
    prefill_only = args.workload == "prefill"
    tp = world
    n_exp = args.experts or E
    # weights: the full layer from one seed on every rank (then this rank's intermediate shard)
    w = synthetic.make_layer_weights(H, n_exp, INTER, SHARED, seed=1, device=dev)
    suffix = f"_e{n_exp}" if n_exp != E else ""
    hbm, _, _ = peaks()

    if tp == 1 and prefill_only:
        tokens = args.tokens or 8192
        x = synthetic.make_hidden(tokens, H, seed=2, device=dev)
        r = time_layer(args, lib, dev, w, x, tokens=tokens, n_exp=n_exp)
        roof, dom = roofline(r, tokens, prefill=True)
        res = base_line(args, world, r, tokens, n_exp, tp, f"prefill_c2{suffix}", prefill=True)
        res.update({"roofline": dict(roof, traffic=traffic_for(f"prefill_c2{suffix}", dom)),
                    "layer": layer_summary(r, tokens, tp, None, False), "e2e": r.get("e2e"),
                    "cpu_baseline": None})
        if rank == 0:
            emit(res)
        return

    if tp == 1:
        # BASELINE config 1 (the headline line), then config 2 on the same layer (the prefill object)
        tokens = args.tokens or 64
        x = synthetic.make_hidden(tokens, H, seed=2, device=dev)
        logits = synthetic.uniform_logits(tokens, n_exp, seed=3, device=dev)
        r = time_layer(args, lib, dev, w, x, tokens=tokens, n_exp=n_exp, logits=logits)
        roof, dom = roofline(r, tokens, prefill=False)
        workload = f"decode_c1{suffix}"
        res = base_line(args, world, r, tokens, n_exp, tp, workload, prefill=False)
        res.update({"roofline": dict(roof, traffic=traffic_for(workload, dom)),
                    "layer": layer_summary(r, tokens, tp, None, False), "e2e": r.get("e2e")})
        if not args.no_prefill:
            pt = 8192
            px = synthetic.make_hidden(pt, H, seed=4, device=dev)
            pr = time_layer(args, lib, dev, w, px, tokens=pt, n_exp=n_exp)
            proof, pdom = roofline(pr, pt, prefill=True)
            pl = layer_summary(pr, pt, tp, None, False)
            res["prefill"] = {
                "workload": f"prefill_c2{suffix}", "tokens": pt, "value": pr["value"], "unit": "tokens/s",
                "ms_per_step": pr["ms_step"], "steps": args.steps, "warmup": args.warmup,
                "router": "from the hidden states inside every timed step (tcgen05 router GEMM + top-k)",
                "roofline": dict(proof, traffic=traffic_for(f"prefill_c2{suffix}", pdom)),
                "layer": pl, "fp8_tflops": pl["fp8_tflops"],
                "fp8_frac": pl["fp8_tflops"] / (2 * peaks()[1]),
                "hbm_frac_layer": pl["hbm_frac"], "gpu_launches": pr["n_launches"], "clocks": pr["clocks"],
                "e2e": pr.get("e2e"),
                "l2": f"no flush: each step streams {layer_bytes(pr['n_touched'], pr['inter'], pr['shared'], pt) / 1e9:.2f}"
                      " GB of expert weights (> 126 MB L2)"}
            del px
        res["cpu_baseline"] = None if args.no_cpu_baseline else cpu_baseline(x, logits, w, tokens=min(tokens, 64))
        if rank == 0:
            emit(res)
        return

    # N > 1: BASELINE config 3 at TP = N.  First the same 256-token layer unsharded on each
    # rank's own GPU (the same-config 1-GPU point of the scaling curve), then the TP run.
    tokens = args.tokens or 256
    x = synthetic.make_hidden(tokens, H, seed=2, device=dev)
    logits = synthetic.uniform_logits(tokens, n_exp, seed=3, device=dev)
    one = time_layer(args, lib, dev, w, x, tokens=tokens, n_exp=n_exp, logits=logits, want_e2e=False)
    w = shard_moe_weights(w, tp, rank, "inter")
    w = {k: v for k, v in w.items() if torch.is_tensor(v)}
    torch.cuda.empty_cache()
    comm = None
    if not args.nccl_allreduce:
        from muserve_b200 import distributed as D
        comm = D.init_fused_allreduce(tokens, H, required=False)  # None: the peers could not be mapped
    r = time_layer(args, lib, dev, w, x, tokens=tokens, n_exp=n_exp, logits=logits, tp=tp, comm=comm)
    roof, dom = roofline(r, tokens, prefill=False)
    workload = f"tp{tp}_decode_c3{suffix}"
    res = base_line(args, world, r, tokens, n_exp, tp, workload, prefill=False)
    res.update({"roofline": dict(roof, traffic=traffic_for(workload, dom)),
                "layer": layer_summary(r, tokens, tp, comm, args.nccl_allreduce,
                                       combine_alone_ms=one["stage_ms"]["combine"]),
                "e2e": r.get("e2e"), "cpu_baseline": None,
                "same_config_1gpu": {
                    "workload": f"decode_t{tokens}_1gpu{suffix}", "value": one["value"], "unit": "tokens/s",
                    "ms_per_step": one["ms_step"], "combine_ms": one["stage_ms"]["combine"],
                    "how": "the same unsharded layer and 256-token batch on one GPU, timed on every rank's own "
                           "GPU before the TP run (max over ranks)"},
                "efficiency_same_config": r["value"] / (tp * one["value"]),
                "note": "the driver's N=1 point is BASELINE config 1 (64 tokens); efficiency against it mixes "
                        "configs, efficiency_same_config uses the 256-token layer on one GPU"})
    if rank == 0:
        emit(res)


def base_line(args, world, r, tokens, n_exp, tp, workload, *, prefill):
    return {
        "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 acc, bf16 io",
        "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) block-quantised weights, " +
                ("router GEMM from the hidden states)" if prefill else "uniform random router logits)"),
        "config": {"workload": workload, "tokens": tokens, "hidden": H, "experts": n_exp, "top_k": K_TOP,
                   "inter_per_rank": r["inter"], "shared_inter_per_rank": r["shared"], "tp": tp,
                   "parallelism": f"tp{tp}" if tp > 1 else "single",
                   "l2": f"no flush: each step streams "
                         f"{layer_bytes(r['n_touched'], r['inter'], r['shared'], tokens) / 1e9:.2f}"
                         " GB of expert weights (> 126 MB L2)"},
        "gpu_launches": r["n_launches"],
        "clocks": r["clocks"],
    }


def run_stack(args, world, rank, local):
    """the 60-layer MoE-only decode stack at TP=N (the decoder's MoE half per
    layer, attention/GDN taken as identity): ``h <- h + moe_l(rms_norm_gemma(h))`` with the
    router from the normed hidden states, a Zipf(1.2) expert-popularity prior added to each
    layer's router logits, the intermediate sharded over the ranks and one NCCL all-reduce per
    layer.  The whole step is one CUDA graph.  Layers that do not fit in this GPU's memory are
    dropped (the line reports how many ran)."""
    from muserve_b200 import _lib, moe, synthetic
    from muserve_b200.graph import GraphedMoEStack
    lib = _lib.load()
    dev = torch.device("cuda", local)
    tp = world
    tokens = args.tokens or 128
    inter, shared = INTER // tp, SHARED // tp
    per_layer = (E + 1) * expert_bytes(inter) + E * H * 2 + 4 * H + 4 * E
    free, _ = torch.cuda.mem_get_info(dev)
    fit = int((free - 16e9) // per_layer)
    n_layers = int(-max_over_ranks(-float(min(args.layers, fit))))
    if n_layers < 1:
        raise RuntimeError("no layer fits in GPU memory")
    layers, biases = [], []
    for li in range(n_layers):
        # this rank's shard of layer li; the router, the shared-expert gate and the norm weight
        # are the same on every rank (rank-independent seed)
        w = synthetic.make_layer_weights(H, E, inter, shared, seed=10_000 + 100 * li + rank, device=dev)
        g = torch.Generator(device=dev).manual_seed(20_000 + li)
        w["moe.gate.weight"] = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w["moe.shared_expert_gate.weight"] = (torch.randn(1, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w["post_attention_layernorm.weight"] = (torch.randn(H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        layers.append(w)
        biases.append(synthetic.zipf_bias(E, 1.2, seed=30_000 + li, device=dev))
    torch.cuda.synchronize()
    barrier()
    x = synthetic.make_hidden(tokens, H, seed=2, device=dev)
    fused = False
    if tp > 1 and not args.nccl_allreduce:
        from muserve_b200 import distributed as D
        # moe_forward then sums over the group in its combine (None: the peers could not be mapped)
        fused = D.init_fused_allreduce(tokens, H, required=False) is not None
    stack = GraphedMoEStack(layers, batch_size=tokens, top_k=K_TOP, device=dev, norm=True, logit_biases=biases)
    # routing statistics and this library's launches per step, from one eager step
    routing = []
    n0 = moe.launch_count()
    stack.eager(x, routing=routing)
    launches_per_step = moe.launch_count() - n0
    torch.cuda.synchronize()
    touched = [int((torch.bincount(ids.flatten().long(), minlength=E) > 0).sum().item()) for ids in routing]
    top_share = statistics.mean(
        float(torch.bincount(ids.flatten().long(), minlength=E).max().item()) / ids.numel() for ids in routing)
    stack.capture(x)
    stream = torch.cuda.current_stream(dev)  # replays, timing events and copies all run here
    try:
        for _ in range(args.warmup):
            stack.run(x)
        torch.cuda.synchronize()
        _lib.check(lib.msv_check_device_error(stream.cuda_stream), "warmup")
        barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        stack.graph.replay()
        w1.record(stream)
        torch.cuda.synchronize()
        est_ms = max(w0.elapsed_time(w1), 1e-3)
        n_soak = int(max_over_ranks(min(2000, max(0, int(args.clock_window_ms / est_ms) - args.steps))))
        barrier()
        torch.cuda.synchronize()
        with Clocks(local) as clk:
            clk.mark(True)
            for _ in range(n_soak):
                stack.graph.replay()
            t0.record(stream)
            for _ in range(args.steps):
                stack.graph.replay()
            t1.record(stream)
            torch.cuda.synchronize()
            clk.mark(False)
        barrier()
        ms_total = max_over_ranks(t0.elapsed_time(t1))
        _lib.check(lib.msv_check_device_error(stream.cuda_stream), "timed region")
        # e2e through the public API: pinned host input copied in, output read back, every step
        e2e = None
        if not args.no_e2e:
            hx = x.cpu().pin_memory()
            ho = torch.empty(tokens, H, dtype=torch.bfloat16).pin_memory()
            dx = torch.empty_like(x)

            def e2e_step():
                dx.copy_(hx, non_blocking=True)
                o = stack.run(dx)
                ho.copy_(o, non_blocking=True)
            for _ in range(args.warmup):
                e2e_step()
            barrier()
            torch.cuda.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            a1.record(stream)
            torch.cuda.synchronize()
            barrier()
            ms_e2e = max_over_ranks(a0.elapsed_time(a1))
            e2e = {"value": tokens * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                   "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": ho.numel() * 2,
                   "ms_per_step": ms_e2e / args.steps}
    finally:
        stack.close()  # the graph holds NCCL calls: release it before the process group goes
    ms_step = ms_total / args.steps
    hbm, _, peak_kind = peaks()
    step_bytes = sum(n * expert_bytes(inter) for n in touched) + n_layers * (
        expert_bytes(shared) + E * H * 2 + 4 * tokens * H * 2)
    gbs = step_bytes / (ms_step / 1e3) / 1e9
    res = {
        "metric": "60-layer MoE decode stack tokens/s", "value": tokens * args.steps / (ms_total / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 acc, bf16 io",
        "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) block-quantised weights, Zipf(1.2) logit prior)",
        "config": {"workload": f"stack{n_layers}_tp{tp}_c4", "layers": n_layers, "layers_requested": args.layers,
                   "tokens": tokens, "hidden": H, "experts": E, "top_k": K_TOP, "inter_per_rank": inter,
                   "tp": tp, "parallelism": f"tp{tp}" if tp > 1 else "single",
                   "graph": "one CUDA graph per step (norm, router GEMM, top-k, dispatch, quantise, 2 GEMMs, "
                            "combine + all-reduce per layer)",
                   "allreduce": "none" if tp == 1 else ("fused into the combine (peer memory)" if fused else "nccl"),
                   "l2": f"no flush: each step streams {step_bytes / 1e9:.1f} GB per rank (> 126 MB L2)"},
        "step": {"ms": ms_step, "ms_per_layer": ms_step / n_layers, "hbm_gbs": gbs, "hbm_frac": gbs / hbm,
                 "peak_kind": peak_kind, "mean_touched_experts": statistics.mean(touched),
                 "mean_top_expert_share": top_share},
        "roofline": {"bound": "hbm", "kernel": "whole step (graph)", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "peak_kind": peak_kind, "traffic": None},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": dict(clk.summary(), window=f"timed region + {n_soak} identical untimed steps just before it"),
        "e2e": e2e,
        "cpu_baseline": None,
    }
    if rank == 0:
        emit(res)


def cpu_baseline(x, logits, w, tokens):
    """The reference's algorithm on the host cores (the CPU oracle port, all threads), on
    ``tokens`` tokens of the same workload with their GPU routing.  Only the touched routed
    experts are copied to the host."""
    from oracle import moe_oracle as orc
    torch.set_num_threads(os.cpu_count())
    xs = x[:tokens].cpu()
    tw, tid = orc.route(logits[:tokens].cpu(), K_TOP)
    shared = {k: v.cpu() for k, v in w.items() if k.startswith("moe.shared")}
    experts = sorted(set(tid.flatten().tolist()))
    cache = {}
    for e in experts:
        cache[e] = (torch.cat([w["moe.experts.gate_proj.weight"][e], w["moe.experts.up_proj.weight"][e]]).cpu(),
                    torch.cat([w["moe.experts.gate_proj.weight_scale_inv"][e],
                               w["moe.experts.up_proj.weight_scale_inv"][e]]).cpu(),
                    w["moe.experts.down_proj.weight"][e].cpu(), w["moe.experts.down_proj.weight_scale_inv"][e].cpu())
    t = time.perf_counter()
    orc.moe_forward_tokens(xs, shared, tw, tid, expert_fn=lambda e: cache[e])
    dt = time.perf_counter() - t
    return {"value": tokens / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{tokens} tokens of the same layer ({len(experts)} experts touched), one pass, "
                      f"{dt:.1f} s"}


def run_reference(args, world, rank):
    """--impl reference: the reference's algorithm on the box's host cores, on the same layer
    (the same seeded weights as our arm, copied to the host) and the same batch, every step the
    whole batch: the CPU oracle port of ``qwen35_layer_v2.moe_forward`` (router softmax/top-k,
    permutation, per-128 quantisation, the two block-scaled GEMMs expert by expert, unsort,
    combine, shared expert), which is pinned bit for bit against the reference's own
    ``moe_forward`` around the GEMMs.  The reference itself imports the MUSA-only
    ``torch_musa`` and ``mate`` and cannot run here.  Under torchrun only rank 0 runs."""
    if rank != 0:
        return
    from muserve_b200 import synthetic
    from muserve_b200.loader import fuse_gate_up
    from oracle import moe_oracle as orc
    torch.set_num_threads(os.cpu_count())
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    tokens = args.tokens or (64 if world == 1 else 256)  # the config our arm runs at this N
    workload = "decode_c1" if world == 1 else f"tp{world}_decode_c3"
    n_exp = args.experts or E
    w = synthetic.make_layer_weights(H, n_exp, INTER, SHARED, seed=1, device=dev)
    x = synthetic.make_hidden(tokens, H, seed=2, device=dev).cpu()
    logits = synthetic.uniform_logits(tokens, n_exp, seed=3, device=dev).cpu()
    # weight preparation is not timed: host copy, and gate/up fused once as the reference does
    # lazily on its first call (qwen35_layer_v2.py:543-558)
    wc = fuse_gate_up({k: v.cpu() for k, v in w.items()})
    del w
    if dev.type == "cuda":
        torch.cuda.empty_cache()

    def step():
        orc.moe_forward(x, wc, n_exp, K_TOP, logits=logits)
    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t
    value = tokens * args.steps / dt
    sample = (f"all {tokens} tokens every step (the whole batch), whole layer on one host"
              + ("" if world == 1 else " (the TP split does not apply to one CPU)")
              + f", torch CPU, {os.cpu_count()} threads")
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 dequantised to fp32 (torch CPU)",
        "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) block-quantised weights, uniform random router logits)",
        "config": {"workload": workload + (f"_e{n_exp}" if n_exp != E else ""), "tokens": tokens, "hidden": H,
                   "experts": n_exp, "top_k": K_TOP,
                   "inter_per_rank": INTER // world, "shared_inter_per_rank": SHARED // world, "tp": world,
                   "parallelism": f"tp{world}" if world > 1 else "single"},
        "same_config": True,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


# The result line is the only thing this script writes to stdout: libraries that print there
# (NCCL's version banner when NCCL_DEBUG asks for it, at communicator creation) write to
# stderr instead, because fd 1 points at stderr while the script runs.
_RESULT_FD = None


def _claim_stdout() -> None:
    global _RESULT_FD
    if _RESULT_FD is None:
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(obj: dict) -> None:
    line = (json.dumps(obj) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, line)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "stack"])
    ap.add_argument("--layers", type=int, default=60, help="layers of the stack workload")
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--experts", type=int, default=0, help="smaller expert count, for profiler captures only")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="TP: plain combine + NCCL all-reduce instead of the fused peer-memory combine")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="N=1: skip the config-2 prefill object")
    ap.add_argument("--clock-window-ms", type=float, default=500.0,
                    help="length of the clock-sampling window (0: timed region only, for profiler runs)")
    args = ap.parse_args()
    _claim_stdout()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = setup_dist()
    try:
        if args.workload == "stack":
            run_stack(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if dist.is_initialized():
            from muserve_b200 import distributed as D
            D.close_fused_allreduce()  # unmaps the peers' buffers (collective)
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
