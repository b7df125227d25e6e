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

``loss_fn`` returns either a scalar loss or a pair ``(output, grad_output)``
for a backward seeded with an explicit output gradient.

Rules that come with graph replay:
* Shapes and dtypes of the batch tensors must stay the same (they are copied
  into static buffers before each replay; with ``static_inputs=True`` the
  example tensors themselves are the graph's inputs and calls must pass those
  same tensors, refilled in place by the caller).
* Gradients live in fixed buffers the graph writes: do not set them to None
  between steps (``optimizer.zero_grad(set_to_none=True)``); each replay
  overwrites them.
* A ladder escalation changes a layer's working dtype and buffers: the step
  is captured again on the next call (escalations are rare).
* The first ``warmup`` calls run eagerly (they are real steps), then the
  capture happens on a side stream.

Data parallel: the gradient reductions are captured on a forked stream (they
overlap the backward kernels that follow them inside the graph), and the
ladder decision of each step waits only for the step's compute (an event the
graph records before it joins the reductions), so the decision and the bulk
reduction overlap too; the caller's stream waits for both before anything
that follows (the optimizer step, the next replay).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch


class GraphedTrainStep:
    def __init__(self, manager, loss_fn: Callable[..., torch.Tensor], example_batch: Sequence[torch.Tensor],
                 warmup: int = 3, static_inputs: bool = False):
        self.mgr = manager
        self.loss_fn = loss_fn
        self.static_inputs = static_inputs
        self.static = list(example_batch) if static_inputs else [t.detach().clone() for t in example_batch]
        self.warmup = max(1, warmup)
        self.calls = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.static_loss: Optional[torch.Tensor] = None
        self.levels: Optional[List[int]] = None
        self.captures = 0
        self.captured_launches = 0
        self.ev_compute = None      # recorded by the graph when the step's compute is done
        self.ladder_stream = None
        self.params = [p for p in manager.model.parameters() if p.requires_grad]

    def _levels(self):
        return [m.level for m in self.mgr.apa_modules.values()]

    @staticmethod
    def _backward(out):
        if isinstance(out, (tuple, list)):
            torch.autograd.backward(out[0], out[1])
            return out[0]
        out.backward()
        return out

    def _eager(self, batch):
        self.mgr.pre_step()
        loss = self._backward(self.loss_fn(*batch))
        keep = self.mgr.post_backward_sync_and_eval()
        return loss.detach(), keep

    def _capture(self):
        dev = self.static[0].device
        # gradients must be produced (not accumulated) by the captured backward,
        # for the parameters and for inputs that require grad
        for p in self.params:
            p.grad = None
        for t in self.static:
            if t.requires_grad:
                t.grad = None
        from . import _lib
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        calls0 = _lib.calls
        dp = getattr(self.mgr, "_dp", None)
        ev = torch.cuda.Event(external=True) if dp is not None else None
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                self.mgr.pre_step()
                loss = self._backward(self.loss_fn(*self.static))
                if dp is not None:
                    ev.record(side)
                    dp.join_capture(side)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.ev_compute = ev
        if dp is not None:
            dp.graph_captured()
        self.graph = g
        self.captured_launches = _lib.calls - calls0   # library launches inside one replay
        self.static_loss = loss.detach()
        self.levels = self._levels()
        self.captures += 1

    def __call__(self, *batch: torch.Tensor) -> Tuple[torch.Tensor, bool]:
        self.calls += 1
        if self.calls <= self.warmup:
            return self._eager(batch)
        for dst, src in zip(self.static, batch):
            if self.static_inputs:
                if src is not dst:
                    raise ValueError("static_inputs: pass the example tensors themselves")
            else:
                dst.copy_(src, non_blocking=True)
        if self.graph is None or self._levels() != self.levels:
            self.graph = None
            torch.cuda.synchronize()
            self._capture()
        self.graph.replay()
        if self.ev_compute is not None:
            cur = torch.cuda.current_stream(self.static[0].device)
            if self.ladder_stream is None:
                self.ladder_stream = torch.cuda.Stream(device=self.static[0].device)
            self.ladder_stream.wait_event(self.ev_compute)
            with torch.cuda.stream(self.ladder_stream):
                keep = self.mgr.post_backward_sync_and_eval()
            cur.wait_stream(self.ladder_stream)
        else:
            keep = self.mgr.post_backward_sync_and_eval()
        return self.static_loss, keep
