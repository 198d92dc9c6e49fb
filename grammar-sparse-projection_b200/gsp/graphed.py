"""The grammar-conditioned LM head as one CUDA graph: the device-side mask path.

The reference's decode loop (benchmarks/qwen35_adaptive_paired.py:46-110)
fills a pinned bitmask on the CPU (xgrammar), copies it to the GPU
(gsp/triton_runtime.py:133-144), picks a route on the host from a CPU
full-word fraction (gsp/triton_runtime.py:310-353) and launches the head.
Here the mask copy runs on its own stream and the head is one graph replay
with no host decision and no host wait:

  stage_mask()  host-to-device copy of the pinned mask on a copy stream,
                issued as soon as the grammar matcher has filled it, so it
                overlaps the transformer layers running on the compute stream;
  step()        the compute stream waits for that copy (an event, no host
                wait) and replays the graph: the route selector kernel (exact
                legal-token and active-tile counts of this step's mask, the
                B200 cost model, cudaGraphSetConditional on a SWITCH node) and
                the chosen projection (row-sparse, block-sparse or dense-mask)
                with the fused greedy top-1 and, when asked for, the masked
                logits.

Before refilling mask_host for the next step, call wait_mask_copied() (the
previous copy has long finished by then in a decode loop; this only guards
the buffer).
"""
from __future__ import annotations

import torch

from . import _native
from .triton_runtime import HeadResult, allocate_pinned_bitmask, grammar_head


class GraphedGrammarHead:
    """Static-buffer grammar head captured once, replayed every decode step.

    weight: CUDA [V, H] float16/bfloat16 LM-head weight. batch: requests per
    step. Buffers: `hidden` (device [B, H], written by the caller or by
    step(hidden)), `mask_host` (pinned [B, ceil(V/32)] int32, filled by the
    grammar matcher; starts all legal), `mask` (its device copy), and `out`
    (HeadResult: logits or None, top_value, top_index, route). cost overrides
    fields of the route cost model (gsp_route_cost).
    """

    def __init__(self, weight: torch.Tensor, batch: int, *, return_logits: bool = True,
                 cost: dict | None = None):
        if weight.device.type != "cuda" or weight.ndim != 2:
            raise ValueError("weight must be a CUDA [V, H] tensor")
        _native.dtype_code(weight.dtype)
        if weight.dtype == torch.float32:
            raise ValueError("GraphedGrammarHead takes float16 or bfloat16 weights")
        if batch < 1:
            raise ValueError("batch must be positive")
        dev = weight.device
        vocab, hidden_dim = weight.shape
        self.weight = weight
        self.batch = batch
        self.cost = cost
        self.hidden = torch.zeros(batch, hidden_dim, dtype=weight.dtype, device=dev)
        self.mask_host = allocate_pinned_bitmask(batch, vocab)
        self.mask = torch.empty(self.mask_host.shape, dtype=torch.int32, device=dev)
        self.out = HeadResult(
            torch.empty(batch, vocab, dtype=weight.dtype, device=dev) if return_logits else None,
            torch.empty(batch, dtype=torch.float32, device=dev),
            torch.empty(batch, dtype=torch.int64, device=dev),
            torch.zeros(1, dtype=torch.int32, device=dev))
        self.copy_stream = torch.cuda.Stream(dev)
        self.copied = torch.cuda.Event()
        self._staged = False        # a copy the next step must wait for
        self._copy_pending = False  # a copy mask_host may still be read by
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            # Warm-up on the capturing stream: every route once (kernel
            # attributes, this stream's workspace), then the head itself.
            self.mask.copy_(self.mask_host, non_blocking=True)
            o = self.out
            _native.row_sparse(self.hidden, weight, self.mask, logits=o.logits, top_value=o.top_value,
                               top_index=o.top_index)
            if batch >= 2:
                _native.block_gemm(self.hidden, weight, self.mask, logits=o.logits, top_value=o.top_value,
                                   top_index=o.top_index)
                _native.dense_masked(self.hidden, weight, self.mask, logits=o.logits, top_value=o.top_value,
                                     top_index=o.top_index)
            grammar_head(self.hidden, weight, self.mask, cost=cost, out=self.out)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            grammar_head(self.hidden, weight, self.mask, cost=cost, out=self.out)

    def stage_mask(self) -> None:
        """Enqueue the host-to-device copy of mask_host on the copy stream
        (after the work already queued on the current stream that last read
        the device mask)."""
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.weight.device))
        with torch.cuda.stream(self.copy_stream):
            self.mask.copy_(self.mask_host, non_blocking=True)
            self.copied.record(self.copy_stream)
        self._staged = True
        self._copy_pending = True

    def wait_mask_copied(self) -> None:
        """Host wait until the last staged copy has read mask_host."""
        if self._copy_pending:
            self.copied.synchronize()
            self._copy_pending = False

    def step(self, hidden: torch.Tensor | None = None) -> HeadResult:
        """One head step on the current stream: waits (on the device) for the
        staged mask copy, copies `hidden` into the static buffer when given,
        then replays the graph (route choice, projection). Outputs are in
        self.out (read them after the stream reaches this point; the next step
        overwrites them)."""
        cur = torch.cuda.current_stream(self.weight.device)
        if self._staged:
            cur.wait_event(self.copied)
            self._staged = False
        if hidden is not None:
            self.hidden.copy_(hidden)
        self.graph.replay()
        return self.out

    def route_names(self) -> list[str]:
        """Names of the routes the last step took (reads the device: synchronises)."""
        from .triton_runtime import ROUTES
        return [ROUTES[int(r)] for r in self.out.route.tolist()]
