"""Whole-step CUDA-graph capture of an energy / forces / stress evaluation.

An E+F+S step launches several hundred kernels (the operators' kernels plus the
element-wise glue of the model and its autograd backward); on the host that is ~25 ms of
Python dispatch per step, which at 4-8 GPUs per cell exceeds the GPU work. Capturing the
step once and replaying it removes the host cost; the graph reads its inputs from static
device buffers, so a new step copies new positions (and, for a new structure of the same
shape, cell / types / edges) into those buffers and replays.

Requirements the captured step meets: fixed tensor shapes (one structure, one edge count,
one domain plan), no host synchronisation inside the step (``use_shifts`` is given as a
Python bool so the periodic-shift test needs no device read), device allocations from the
torch caching allocator or the operators' stream-ordered pool (which capture turns into
graph allocation nodes), and, across GPUs, NCCL collectives issued in the same order on
every rank (captured like kernels).
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Optional

import torch


class GraphedStep:
    """``fn(inputs) -> dict of tensors`` captured into a CUDA graph.

    ``example`` holds the inputs of the capture: its tensors become the static buffers
    (cloned), other values are passed through unchanged. Calling the object copies any
    given tensors into the static buffers (same shapes) and replays the graph; it returns
    the static output dict, valid until the next call.
    """

    def __init__(self, fn: Callable[[Dict[str, Any]], Dict[str, torch.Tensor]], example: Dict[str, Any],
                 warmup: int = 2):
        self.fn = fn
        self.static = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in example.items()}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                fn(self.static)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn(self.static)

    def __call__(self, inputs: Optional[Dict[str, torch.Tensor]] = None) -> Dict[str, torch.Tensor]:
        if inputs:
            for k, v in inputs.items():
                self.static[k].copy_(v, non_blocking=True)
        self.graph.replay()
        return self.out

    def release(self) -> None:
        """Free the graph (before destroying a process group whose collectives it holds)."""
        self.graph.reset()
        self.out = None
