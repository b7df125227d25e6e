"""AdamW whose update of every APALinear weight also writes that layer's next
working copy.

The reference trains with ``torch.optim.AdamW(manager.get_trainable_parameters())``
and then re-casts every master weight in ``pre_step`` (manager.py:145-172,
layers.py:368-372): the optimizer reads and writes p, grad, m, v and the
refresh reads p again to write the working copies. ``APAAdamW`` does both in
one pass per weight (``apa_adamw_cast``: p, g, m, v arrive by TMA tiles, p, m and v are updated
in place and stored back, and the updated master is cast to the layer's
working dtype, with its transposed copy when the backward needs it, while it
is still in registers); the weight's telemetry comes along and the following
``pre_step`` skips that layer's weight cast. Every other parameter (biases,
LayerNorm, embeddings) and any weight the fused kernel cannot take goes
through torch's fused AdamW (its step counters then live on the device). Semantics are those of
``torch.optim.AdamW`` (decoupled weight decay, no amsgrad); results agree to
fp32 rounding.

    opt = APAAdamW(manager, lr=1e-3, weight_decay=0.01)
    ...
    if manager.post_backward_sync_and_eval():
        opt.step()
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch
from torch.optim import adamw as _torch_adamw

from . import _lib


class APAAdamW(torch.optim.Optimizer):
    def __init__(self, manager, lr: float = 1e-3, betas: Tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2):
        super().__init__(manager.get_trainable_parameters(),
                         dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.mgr = manager
        self._owner: Dict[int, object] = {id(m.weight_master): m for m in manager.apa_modules.values()}
        self.fused_steps = 0        # weight updates done by the fused kernel (for tests and reports)

    def _state(self, p, fused_weight: bool):
        st = self.state[p]
        if not st:
            # the fused weight kernel counts steps on the host; every other
            # parameter goes through torch's fused AdamW, which wants its step
            # counter on the parameter's device
            st["step"] = torch.zeros((), dtype=torch.float32, device="cpu" if fused_weight else p.device)
            st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return st

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr = float(group["lr"])
            beta1, beta2 = group["betas"]
            eps, wd = float(group["eps"]), float(group["weight_decay"])
            rest = ([], [], [], [], [])
            for p in group["params"]:
                if p.grad is None:
                    continue
                mod = self._owner.get(id(p))
                st = self._state(p, mod is not None)
                if mod is not None:
                    n = (st["fused_step"] if "fused_step" in st else int(st["step"].item())) + 1
                    if mod._adamw_refresh(p, p.grad, st["exp_avg"], st["exp_avg_sq"], lr, beta1, beta2, eps, wd, n):
                        st["fused_step"] = n
                        st["step"].fill_(n)
                        self.fused_steps += 1
                        continue
                    st.pop("fused_step", None)   # the regular path counts the step itself
                if p.is_cuda and st["step"].device != p.device:
                    st["step"] = st["step"].to(p.device)
                rest[0].append(p)
                rest[1].append(p.grad)
                rest[2].append(st["exp_avg"])
                rest[3].append(st["exp_avg_sq"])
                rest[4].append(st["step"])
            if rest[0]:
                fused = all(t.is_cuda and t.dtype == torch.float32 for t in rest[0]) or None
                _torch_adamw.adamw(rest[0], rest[1], rest[2], rest[3], [], rest[4], fused=fused, amsgrad=False,
                                   beta1=beta1, beta2=beta2, lr=lr, weight_decay=wd, eps=eps, maximize=False)
        return loss
