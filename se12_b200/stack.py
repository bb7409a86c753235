"""A decode step's GEMVs as one replayable CUDA graph.

``GemvStack`` records a sequence of fused SE12 GEMVs (matrix, input
buffer, output buffer), runs them eagerly or captures them once into a CUDA
graph and replays it. Kernels are launched with programmatic dependent
launch, so inside the graph each GEMV's CTAs start fetching weights while
the previous GEMV drains. This is the stacked mode of the reference's
microbenchmark design (the same projections of every layer back to back in
one graph), used by the benchmark and by the runtime.
"""

from __future__ import annotations

import dataclasses

import torch

from .device import DeviceSe12Matrix, bf16_gemv, gemv_call


@dataclasses.dataclass
class GemvOp:
    matrix: DeviceSe12Matrix | None  # None: dense BF16 baseline with `weights`
    x: torch.Tensor
    y: torch.Tensor
    weights: torch.Tensor | None = None


class GemvStack:
    """With ``chain=True`` the sequence runs as one persistent launch
    (``se12_b200.chain.Se12Chain``: op j reads x once op j - 1 is done, the
    next op's weights stream in meanwhile) instead of one launch per GEMV;
    every op then needs the same batch, and SE12 and dense ops do not mix."""

    def __init__(self, device: torch.device | str = "cuda", chain: bool = False):
        self.device = torch.device(device)
        self.ops: list = []
        self.graph: torch.cuda.CUDAGraph | None = None
        self.stream = torch.cuda.Stream(self.device)
        self.use_chain = bool(chain)
        self.chain = None

    def add(self, matrix: DeviceSe12Matrix, x: torch.Tensor, y: torch.Tensor) -> None:
        self.ops.append(GemvOp(matrix, x, y))
        self.graph = None
        self.chain = None

    def add_dense(self, weights: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> None:
        self.ops.append(GemvOp(None, x, y, weights))
        self.graph = None
        self.chain = None

    @property
    def launches(self) -> int:
        return 1 if self.use_chain else len(self.ops)

    def _build_chain(self):
        from .chain import Se12Chain

        dense = self.ops[0].matrix is None
        batch = self.ops[0].x.shape[0]
        chain = Se12Chain(batch, self.device, dense=dense)
        for op in self.ops:
            if (op.matrix is None) != dense or op.x.shape[0] != batch:
                raise ValueError("a chain needs one batch size and one kind of GEMV")
            if dense:
                chain.add_dense(op.weights, op.x, op.y)
            else:
                chain.add(op.matrix, op.x, op.y)
        chain.upload()
        self.chain = chain

    def _launch_all(self) -> None:
        if self.use_chain:
            if self.chain is None:
                self._build_chain()
            self.chain.run()
            return
        for op in self.ops:
            if op.matrix is not None:
                gemv_call(op.matrix, op.x, op.y)
            else:
                bf16_gemv(op.weights, op.x, op.y)

    def run(self) -> None:
        """Eager launches on the current stream."""
        self._launch_all()

    def capture(self, warmup: int = 1) -> None:
        """Captures the sequence into a CUDA graph on this stack's stream."""
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self._launch_all()
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self._launch_all()
        self.graph = graph

    def replay(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()
