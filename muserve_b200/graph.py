"""A stack of MoE layers captured into one CUDA graph, the counterpart of the reference's
``GraphedDecodeStep`` (``muserve/model/graph_decode.py:23-113``): warm up three times, capture
once, then replay with no per-kernel host work.

Every kernel of the layer takes its sizes from device memory (routing, per-expert counts and
the GEMM tile lists are built on the device), nothing reads back to the host, and the
workspace is reused from the capture stream's cache, so the whole step (router GEMM, the six
layer kernels, the TP all-reduce when one is initialised) records as plain graph nodes.

One step runs each layer's MoE half of the decoder layer with the attention/GDN half taken
as identity (the 60-layer stack benchmark).  With ``norm`` (layers carry
``post_attention_layernorm.weight``) a layer is ``h <- h + moe_l(rms_norm_gemma(h))``, as the
reference's decode layer (``qwen35_layer_v2.py:712-715``); the residual add and the next
layer's norm run as one kernel.  Without it a layer is ``x <- x + moe_l(x)`` (``residual``)
or ``x <- moe_l(x)``.  ``logit_biases`` (one [E] fp32 tensor per layer) are added to the
router logits: the expert-popularity prior of the benchmark.  ``run(h)`` copies ``h`` into
the static input and replays; ``step()`` replays on the static buffers and, with
``self_feed``, copies the output back into the input inside the graph (the reference's
self-feeding decode loop).
"""
from __future__ import annotations

import torch

from . import moe
from .model import qwen35_layer_v2 as v2


class GraphedMoEStack:
    def __init__(self, layers: list[dict], batch_size: int, top_k: int, device: torch.device | str | None = None,
                 residual: bool = True, self_feed: bool = False, norm: bool = False,
                 logit_biases: list[torch.Tensor] | None = None, eps: float = 1e-6):
        if not layers:
            raise ValueError("need at least one layer")
        if norm and any("post_attention_layernorm.weight" not in w for w in layers):
            raise ValueError("norm=True needs post_attention_layernorm.weight in every layer")
        if logit_biases is not None and len(logit_biases) != len(layers):
            raise ValueError("one logit bias per layer")
        self.layers = layers
        self.norm = norm
        self.logit_biases = logit_biases
        self.eps = eps
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

    def _bias(self, i: int):
        return None if self.logit_biases is None else self.logit_biases[i]

    def _moe(self, i: int, x: torch.Tensor, routing: list | None) -> torch.Tensor:
        if routing is None:
            return v2.moe_forward(x, self.layers[i], top_k=self.top_k, logit_bias=self._bias(i))
        y, _, ids = v2.moe_forward(x, self.layers[i], top_k=self.top_k, logit_bias=self._bias(i),
                                   return_routing=True)
        routing.append(ids)
        return y

    def eager(self, x: torch.Tensor, routing: list | None = None) -> torch.Tensor:
        """The same step without a graph (warm-up, and the reference for tests).  With a
        ``routing`` list, each layer's top-k ids are appended to it."""
        if self.norm:
            h = x.clone()
            x2 = moe.add_rms_norm_gemma(h, self.layers[0]["post_attention_layernorm.weight"], eps=self.eps)
            for i, w in enumerate(self.layers):
                y = self._moe(i, x2, routing)
                if i + 1 < len(self.layers):
                    x2 = moe.add_rms_norm_gemma(h, self.layers[i + 1]["post_attention_layernorm.weight"], add=y,
                                                eps=self.eps)
                else:
                    moe.add_rms_norm_gemma(h, None, add=y, norm=False)
            return h
        for i in range(len(self.layers)):
            y = self._moe(i, x, routing)
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
