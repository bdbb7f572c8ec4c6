"""CUDA-graph replay of a Newton-Schulz call (the native counterpart of the
reference's compiled torch operation, newton_schulz.py:16-46).

For small matrices the chain's device work is microseconds, so every call is
bounded by launching its kernels (normalisation, then the fused small-matrix
chain or one GEMM launch per product) and by the Python and ctypes work around
them. ``CapturedOrthogonalizer`` records one call on a fixed input buffer as a
CUDA graph and replays it: one host call launches the whole chain.

Semantics follow CUDA-graph replay, as with ``torch.compile``'s CUDA graphs:
the input is copied into the graph's buffer and the returned tensor is the
graph's output buffer, overwritten by the next replay (clone it to keep it).
The capture freezes what the chain reads on the host at capture time: the
coefficients, the small-chain tactic (``ops.small_chain_tactic``) and the
bounded-wait limit; capture again after changing them.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor


class CapturedOrthogonalizer:
    """One orthogonaliser call on tensors shaped like ``example``, replayed from a CUDA graph.

    ``orthogonalizer`` is any callable of this package that runs on the current
    stream (``GramNewtonSchulz``, ``StandardNewtonSchulz``, a fused backend
    operation). Capturing runs it twice eagerly on a side stream (warm-up: the
    first call on a device loads the kernels) and once under capture.
    """

    def __init__(self, orthogonalizer: Callable[[Tensor], Tensor], example: Tensor, warmup: int = 2) -> None:
        if not example.is_cuda:
            raise ValueError("CUDA-graph capture needs a CUDA tensor")
        self.shape = tuple(example.shape)
        self.dtype = example.dtype
        self.device = example.device
        self.static_input = torch.empty_like(example, memory_format=torch.contiguous_format)
        self.static_input.copy_(example)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                orthogonalizer(self.static_input)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_output = orthogonalizer(self.static_input)

    def __call__(self, matrix: Tensor) -> Tensor:
        if tuple(matrix.shape) != self.shape or matrix.dtype != self.dtype or matrix.device != self.device:
            raise ValueError(
                f"captured for {self.shape} {self.dtype} on {self.device}, got "
                f"{tuple(matrix.shape)} {matrix.dtype} on {matrix.device}"
            )
        if matrix.data_ptr() != self.static_input.data_ptr():
            self.static_input.copy_(matrix)
        self.graph.replay()
        return self.static_output

    def replay(self) -> Tensor:
        """Runs the chain on whatever ``static_input`` holds (no copy)."""
        self.graph.replay()
        return self.static_output
