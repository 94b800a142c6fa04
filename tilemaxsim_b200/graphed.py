"""A fixed-shape search step captured once as a CUDA graph and replayed per call.

A search step is a handful of short launches (query packing, the scoring kernel, one or two top-k
kernels); issuing them from Python costs a few hundred microseconds of host time per step, which an
end-to-end caller (queries from host memory in, top-k back to host memory out, every step) pays on
top of the GPU time. Replaying a captured graph issues the whole step with one launch.

    step = GraphedStep(lambda Q: index.search(Q, k), Q_example_on_gpu)
    vals, ids = step(Q_host)          # pinned host tensors, overwritten by the next call

`fn` must launch only stream-ordered GPU work on the current stream and return tensors: every
tilemaxsim_b200 scoring and top-k call qualifies (no host synchronisation, no allocation outside
torch's allocator). Collectives are not captured: this is for one GPU (a capture that fails on one
rank but not on another would leave the other rank's graph waiting in a collective), so a
multi-GPU search runs its steps eagerly.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class GraphedStep:
    def __init__(self, fn: Callable[..., torch.Tensor | Sequence[torch.Tensor]], *example_inputs: torch.Tensor,
                 warmup: int = 2):
        if not example_inputs or any(x.device.type != "cuda" for x in example_inputs):
            raise ValueError("GraphedStep needs CUDA example inputs (their shapes and dtypes are fixed)")
        dev = example_inputs[0].device
        self.device = dev
        self.inputs = [x.detach().clone() for x in example_inputs]
        with torch.cuda.device(dev):
            cur = torch.cuda.current_stream(dev)
            side = torch.cuda.Stream(dev)
            side.wait_stream(cur)
            with torch.cuda.stream(side):  # first calls (lazy initialisation) outside the capture
                for _ in range(max(1, warmup)):
                    fn(*self.inputs)
            cur.wait_stream(side)
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            # thread-local capture: CUDA calls other threads make meanwhile are not restricted
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                out = fn(*self.inputs)
        self.single = isinstance(out, torch.Tensor)
        self.outputs = [out] if self.single else list(out)
        self.host_outputs = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in self.outputs]

    def replay(self, *inputs: torch.Tensor) -> list[torch.Tensor]:
        """Copies `inputs` (host or device, the captured shapes) into the static inputs and replays
        the graph on the current stream; returns the static device outputs (asynchronous)."""
        if len(inputs) != len(self.inputs):
            raise ValueError(f"expected {len(self.inputs)} inputs, got {len(inputs)}")
        with torch.cuda.device(self.device):
            for dst, src in zip(self.inputs, inputs):
                if src.shape != dst.shape:
                    raise ValueError(f"input shape {tuple(src.shape)} != captured {tuple(dst.shape)}")
                dst.copy_(src, non_blocking=True)
            self.graph.replay()
        return self.outputs

    def __call__(self, *inputs: torch.Tensor):
        """replay() plus a copy of every output to pinned host memory; synchronises the stream."""
        outs = self.replay(*inputs)
        with torch.cuda.device(self.device):
            for h, o in zip(self.host_outputs, outs):
                h.copy_(o, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
        return self.host_outputs[0] if self.single else tuple(self.host_outputs)
