"""A stack of MoE layers captured into one CUDA graph, the counterpart of the reference's
``GraphedDecodeStep`` (``muserve/model/graph_decode.py:23-113``): warm up three times, capture
once, then replay with no per-kernel host work.

Every kernel of the layer takes its sizes from device memory (routing, per-expert counts and
the GEMM tile lists are built on the device), nothing reads back to the host, and the
workspace is reused from the capture stream's cache, so the whole step (router GEMM, the six
layer kernels, the TP all-reduce when one is initialised) records as plain graph nodes.

One step is ``x <- x + moe_l(x)`` for each layer ``l`` (the decoder's attention is outside
the path and taken as identity, as in the 60-layer stack benchmark).  ``run(h)`` copies ``h``
into the static input and replays; ``step()`` replays on the static buffers and, with
``self_feed``, copies the output back into the input inside the graph (the reference's
self-feeding decode loop).
"""
from __future__ import annotations

import torch

from .model import qwen35_layer_v2 as v2


class GraphedMoEStack:
    def __init__(self, layers: list[dict], batch_size: int, top_k: int, device: torch.device | str | None = None,
                 residual: bool = True, self_feed: bool = False):
        if not layers:
            raise ValueError("need at least one layer")
        self.layers = layers
        self.batch_size = batch_size
        self.top_k = top_k
        self.device = torch.device(device) if device is not None else layers[0]["moe.gate.weight"].device
        self.hidden = layers[0]["moe.gate.weight"].shape[1]
        self.residual = residual
        self.self_feed = self_feed
        self.graph = None
        self.stream = None
        self.inp = None
        self.out = None

    def eager(self, x: torch.Tensor) -> torch.Tensor:
        """The same step without a graph (warm-up, and the reference for tests)."""
        for w in self.layers:
            y = v2.moe_forward(x, w, top_k=self.top_k)
            x = x + y if self.residual else y
        return x

    def capture(self, sample: torch.Tensor) -> None:
        if sample.shape != (self.batch_size, self.hidden) or sample.dtype != torch.bfloat16:
            raise ValueError(f"sample must be bf16 [{self.batch_size}, {self.hidden}]")
        self.inp = sample.to(self.device).clone()
        self.stream = torch.cuda.Stream(self.device)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            for _ in range(3):
                self.eager(self.inp)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = self.eager(self.inp)
            if self.self_feed:
                self.inp.copy_(self.out)
        torch.cuda.synchronize(self.device)

    def run(self, hidden: torch.Tensor) -> torch.Tensor:
        """Replay on ``hidden``; the result is the graph's static output buffer."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        self.inp.copy_(hidden)
        self.graph.replay()
        return self.out

    def step(self) -> torch.Tensor:
        """Replay on the static input (with ``self_feed``, the previous step's output)."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        self.graph.replay()
        return self.out

    def close(self) -> None:
        """Release the graph (before the process group goes, when it holds collectives)."""
        if self.graph is not None:
            self.graph.reset()
        self.graph = None
        self.out = None
