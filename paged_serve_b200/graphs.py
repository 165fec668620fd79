"""CUDA-graph capture of the decode step's attention loop.

A decode step launches, for each of L layers, one append and one paged-decode
kernel (plus a split-K combine for long contexts). Replaying them from one
captured graph removes the per-launch host cost (Python, ctypes, the driver's
launch path) and most of the gap between dependent kernels. The graph is
captured once for a fixed batch of rows over static metadata
(:meth:`PagedCudaBackend.static_decode_metadata`); each step refills the
metadata in place — one pinned upload plus the device slot builder — and
replays. An engine that captures its whole model forward uses the same
static metadata inside its own capture.
"""

from __future__ import annotations

import torch

from paged_serve_b200.backend import PagedCudaBackend
from paged_serve_b200.block_manager import StepPlan

__all__ = ["DecodeGraph"]


class DecodeGraph:
    """Every layer's decode step (KV append fused into the paged decode) for a static
    batch, as one CUDA graph.

    Write each step's q/k/v into :attr:`query`, :attr:`key`, :attr:`value`
    (``[L, batch, 1, H, D]``), load the step's sequences with :meth:`load_plan`
    or :meth:`load`, then :meth:`replay`; the outputs (``[batch, 1, Hq, D]`` per
    layer) are overwritten in place on each replay.
    """

    def __init__(self, backend: PagedCudaBackend, batch: int, width: int | None = None,
                 layers: int | None = None, timing: bool = False) -> None:
        """``timing``: record an event pair around every layer inside the graph, so
        :meth:`layer_ms` gives each layer's device time in the latest replay."""
        if backend.k_cache is None:
            raise RuntimeError("allocate() the backend before capturing")
        if backend.debug_invariants:
            raise ValueError("graph capture needs debug_invariants off: its checks synchronise")
        m = backend.model
        pools = backend.k_cache.shape[0]
        self.layers = layers or pools
        if self.layers > pools:
            raise ValueError(f"{self.layers} layers but the backend holds {pools} pools")
        self.backend = backend
        self.batch = batch
        self.metadata = backend.static_decode_metadata(batch, width)
        dev, dt = backend.device, backend.dtype
        self.query = torch.zeros((self.layers, batch, 1, m.num_q_heads, m.head_dim), dtype=dt,
                                 device=dev)
        self.key = torch.zeros((self.layers, batch, 1, m.num_kv_heads, m.head_dim), dtype=dt,
                               device=dev)
        self.value = torch.zeros_like(self.key)
        self._events = None
        if timing:
            self._events = [(torch.cuda.Event(enable_timing=True, external=True),
                             torch.cuda.Event(enable_timing=True, external=True))
                            for _ in range(self.layers)]
        # One eager pass first (kernel attributes, tensor-map descriptors), on a side
        # stream as capture requires; with every row inactive it writes nothing.
        main = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            self._body()
        main.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = self._body(capturing=True)

    def _body(self, capturing: bool = False) -> list[torch.Tensor]:
        b, md = self.backend, self.metadata
        outs = []
        for layer in range(self.layers):
            if capturing and self._events:
                self._events[layer][0].record()
            outs.append(b.forward(layer, self.query[layer], self.key[layer], self.value[layer],
                                  md))
            if capturing and self._events:
                self._events[layer][1].record()
        return outs

    def load_plan(self, plan: StepPlan) -> None:
        """The step's sequences from a block-manager plan (block moves run first)."""
        self.backend.load_decode_plan(self.metadata, plan)

    def load(self, block_tables: torch.Tensor, ctx_lens: torch.Tensor) -> None:
        """Sequences whose newest token (at ``ctx_lens - 1``) is this step's."""
        self.backend.load_decode(self.metadata, block_tables, ctx_lens)

    def replay(self) -> list[torch.Tensor]:
        self.graph.replay()
        return self.outputs

    def layer_ms(self) -> list[float]:
        """Device time of each layer (append + decode) in the latest replay (synchronises)."""
        if not self._events:
            raise ValueError("capture with timing=True to time layers")
        torch.cuda.synchronize(self.backend.device)
        return [a.elapsed_time(z) for a, z in self._events]
