"""CUDA-graph replay of a decoder-layer forward.

A layer forward is ~15 kernel launches issued from Python through ctypes;
once the GPU time per layer falls below the host time to issue them, the GPU
idles between kernels.  ``GraphedDecoderLayer`` captures one forward for a fixed
input shape and position ids into a CUDA graph (torch.cuda.CUDAGraph) and
replays it: the same kernels, launched by the driver in one call.

The captured forward reads its input from a static buffer and writes its
outputs to static buffers; ``__call__`` copies the caller's input in, replays,
and returns the static outputs (overwritten by the next call).  Weights are
read where they live: in-place updates are seen by later replays, replacing a
parameter tensor requires a new capture.

With a preallocated ``LayerKVCache`` as ``past_kv`` the captured forward
appends its rows at the cache offset of capture time and attends over that
fixed length: a replay rewrites the same positions and does NOT advance
``cache.length``.  The cache length is restored after the warm-up and the
capture, so the cache reads as it did before construction.  This suits a
fixed-position step (a benchmark); a decode loop needs one capture per
position, or the eager module.
"""
from __future__ import annotations

import torch

from .kv_cache import KVCache, LayerKVCache
from .modules import CudaTextDecoderLayer, TextMRoPE


class GraphedDecoderLayer:
    def __init__(self, layer: CudaTextDecoderLayer, rotary: TextMRoPE, example_x: torch.Tensor,
                 position_ids: torch.Tensor, past_kv=None, warmup: int = 2):
        if not example_x.is_cuda:
            raise RuntimeError("GraphedDecoderLayer: CUDA input required")
        self.layer = layer
        self.static_x = example_x.detach().clone()
        self.static_pos = position_ids.detach().clone()
        if isinstance(past_kv, KVCache):
            raise RuntimeError("GraphedDecoderLayer captures one layer: pass that layer's "
                               "LayerKVCache, not the model's KVCache")
        self.past_kv = past_kv
        length0 = past_kv.length if isinstance(past_kv, LayerKVCache) else None
        bound = rotary.bind(self.static_pos)
        side = torch.cuda.Stream(device=example_x.device)
        side.wait_stream(torch.cuda.current_stream(example_x.device))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(warmup):  # caches (fused weights, TMA attributes) filled outside capture
                if length0 is not None:
                    past_kv.length = length0
                layer(self.static_x, bound, past_kv=past_kv)
        torch.cuda.current_stream(example_x.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        if length0 is not None:
            past_kv.length = length0
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.static_out = layer(self.static_x, bound, past_kv=past_kv)
        if length0 is not None:
            past_kv.length = length0

    def replay(self):
        """Replays the captured forward on the current static input."""
        self.graph.replay()
        return self.static_out

    def __call__(self, x: torch.Tensor):
        """Copies ``x`` into the static input and replays; returns the static
        (x, router_logits, new_kv) of the captured forward."""
        if x.shape != self.static_x.shape:
            raise RuntimeError(f"GraphedDecoderLayer captured shape {tuple(self.static_x.shape)}, "
                               f"got {tuple(x.shape)}")
        self.static_x.copy_(x, non_blocking=True)
        return self.replay()


class StreamedLayerRunner:
    """Runs a GraphedDecoderLayer over a sequence of pinned host inputs with the
    host->device copy of step i+1 and the device->host copy of step i-1
    overlapping the replay of step i (separate copy streams, double-buffered
    device staging).  ``run(x_host, out_host, steps)`` copies ``x_host`` in and
    the layer output back into ``out_host`` on every step."""

    def __init__(self, graphed: GraphedDecoderLayer):
        self.g = graphed
        dev = graphed.static_x.device
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        self.stage_in = [torch.empty_like(graphed.static_x) for _ in range(2)]
        self.stage_out = [torch.empty_like(graphed.static_out[0]) for _ in range(2)]

    def run(self, x_host: torch.Tensor, out_host: torch.Tensor, steps: int) -> None:
        comp = torch.cuda.current_stream(self.g.static_x.device)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_free = [torch.cuda.Event() for _ in range(2)]
        for e in in_free + out_free:
            e.record(comp)

        def load(i):
            b = i % 2
            with torch.cuda.stream(self.h2d):
                self.h2d.wait_event(in_free[b])
                self.stage_in[b].copy_(x_host, non_blocking=True)
                in_ready[b].record(self.h2d)

        load(0)
        for i in range(steps):
            b = i % 2
            if i + 1 < steps:
                load(i + 1)
            comp.wait_event(in_ready[b])
            self.g.static_x.copy_(self.stage_in[b], non_blocking=True)
            in_free[b].record(comp)
            self.g.replay()
            comp.wait_event(out_free[b])
            self.stage_out[b].copy_(self.g.static_out[0], non_blocking=True)
            out_ready[b].record(comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(out_ready[b])
                out_host.copy_(self.stage_out[b], non_blocking=True)
                out_free[b].record(self.d2h)
        comp.wait_stream(self.d2h)
