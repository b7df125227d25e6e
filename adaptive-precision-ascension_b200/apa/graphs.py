"""CUDA-graph replay of a static-shape APA training step.

A training step with many APALinear layers launches a few hundred small
kernels whose host-side issue cost (Python, autograd, ctypes) can exceed the
GPU time. ``GraphedTrainStep`` captures ``APAManager.pre_step()``, the forward
and the backward once into a CUDA graph and replays it every step; the ladder
decision (``post_backward_sync_and_eval``, which needs one host read) stays
eager, as does the optimizer step the caller runs when the step is kept.

    step = GraphedTrainStep(manager, loss_fn, example_batch)
    for batch in data:
        loss, keep = step(*batch)        # replay + ladder decision
        if keep:
            optimizer.step()

Rules that come with graph replay:
* Shapes and dtypes of the batch tensors must stay the same (they are copied
  into static buffers before each replay).
* Gradients live in fixed buffers the graph writes: do not set them to None
  between steps (``optimizer.zero_grad(set_to_none=True)``); each replay
  overwrites them.
* A ladder escalation changes a layer's working dtype and buffers: the step
  is captured again on the next call (escalations are rare).
* The first ``warmup`` calls run eagerly (they are real steps), then the
  capture happens on a side stream.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch


class GraphedTrainStep:
    def __init__(self, manager, loss_fn: Callable[..., torch.Tensor], example_batch: Sequence[torch.Tensor],
                 warmup: int = 3):
        self.mgr = manager
        self.loss_fn = loss_fn
        self.static = [t.detach().clone() for t in example_batch]
        self.warmup = max(1, warmup)
        self.calls = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.static_loss: Optional[torch.Tensor] = None
        self.levels: Optional[List[int]] = None
        self.captures = 0
        self.params = [p for p in manager.model.parameters() if p.requires_grad]

    def _levels(self):
        return [m.level for m in self.mgr.apa_modules.values()]

    def _eager(self, batch):
        self.mgr.pre_step()
        loss = self.loss_fn(*batch)
        loss.backward()
        keep = self.mgr.post_backward_sync_and_eval()
        return loss.detach(), keep

    def _capture(self):
        dev = self.static[0].device
        # gradients must be produced (not accumulated) by the captured backward
        for p in self.params:
            p.grad = None
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                self.mgr.pre_step()
                loss = self.loss_fn(*self.static)
                loss.backward()
        torch.cuda.current_stream(dev).wait_stream(side)
        dp = getattr(self.mgr, "_dp", None)
        if dp is not None:
            dp.graph_captured()
        self.graph = g
        self.static_loss = loss.detach()
        self.levels = self._levels()
        self.captures += 1

    def __call__(self, *batch: torch.Tensor) -> Tuple[torch.Tensor, bool]:
        self.calls += 1
        if self.calls <= self.warmup:
            return self._eager(batch)
        for dst, src in zip(self.static, batch):
            dst.copy_(src, non_blocking=True)
        if self.graph is None or self._levels() != self.levels:
            self.graph = None
            torch.cuda.synchronize()
            self._capture()
        self.graph.replay()
        keep = self.mgr.post_backward_sync_and_eval()
        return self.static_loss, keep
