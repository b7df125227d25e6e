"""APALinear: a drop-in ``nn.Linear`` whose forward and backward run the
B200 kernels of libapa_kernels.so.

Public surface is the reference's (apa/layers.py:10-438): ``APABoundaryCast``,
``APALinear(in_features, out_features, bias=True, config=APAConfig())`` with
``weight_master`` / ``bias_master`` parameters, the persistent buffers
``gpu_amax`` / ``gpu_underflow_ratio`` / ``gpu_has_nonfinite`` (same
state_dict keys), ``level``, ``ema_underflow_ratio``, ``weight_work`` /
``bias_work``, ``working_dtype``, ``refresh_working_copy()``,
``track_telemetry()`` and ``update_underflow_metric()``.

Per step and layer the hot path is (M tokens, K in, N out):

  pre_step     W fp32 -> W_q [N,K] and W_q^T [K,N] in the working dtype, the
               weight's amax kept pending until the forward runs  (1 launch)
  forward      x -> x_q [M,K] (+ x_q^T [K,M] for wgrad), telemetry of x_q and
               the pending weight amax                               (1 launch)
               y = x_q W_q^T + b on tcgen05, telemetry of y          (1 launch)
  backward     dy -> dy_q [M,N] (+ dy_q^T, bias partials), telemetry  (1 launch)
               dx = dy_q W_q  with the engine's re-casts and the boundary
               cast's hook telemetry fused                           (1 launch)
               dW = dy_q^T x_q with underflow counters, written to
               weight_master.grad                                    (1 launch)
               db from the partials                                  (1 launch)

The reference's separate telemetry passes, per-layer ``.item()`` sync and
grad copy to the masters are all folded into those launches.
"""
from __future__ import annotations

import ctypes
import math
import weakref
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from .config import APAConfig, DTYPE_MAP, LEVEL_FP8, LEVEL_FP16, LEVEL_TF32, THRESHOLDS_MIN
from .telemetry import track_telemetry_on_tensor, update_running_underflow

_ROLES = ("input_activation", "weight", "output", "grad_output", "grad_weight", "grad_input")


_ELEM_SIZE = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}
if DTYPE_MAP[LEVEL_FP8] is not None:
    _ELEM_SIZE[DTYPE_MAP[LEVEL_FP8]] = 1


def _elem_size(dtype: torch.dtype) -> int:
    return _ELEM_SIZE[dtype]


def _pad(n: int, es: int) -> int:
    """Smallest m >= n with m * es a multiple of 16 bytes (TMA row pitch)."""
    q = 16 // es
    return ((n + q - 1) // q) * q


def _tma_ok(t: torch.Tensor) -> bool:
    """A 2-D tensor the GEMM can read in place: unit inner stride, 16-byte
    aligned base and row pitch."""
    es = t.element_size()
    return (t.dim() == 2 and t.stride(1) == 1 and t.data_ptr() % 16 == 0
            and (t.stride(0) * es) % 16 == 0)


def _working(level: int) -> torch.dtype:
    return DTYPE_MAP[level] if DTYPE_MAP[level] is not None else torch.float32


def _operand_code(level: int) -> int:
    """C-ABI dtype code of the GEMM operands at a level: the working dtype,
    except that TF32-rung operands are stored rounded to the TF32 grid."""
    return _lib.DT_TF32 if level == LEVEL_TF32 else _lib.dt_code(_working(level))


def _alloc_2d(rows: int, cols: int, dtype: torch.dtype, device) -> torch.Tensor:
    """[rows, cols] view of a buffer whose row pitch is padded to 16 bytes."""
    ld = _pad(cols, _ELEM_SIZE[dtype])
    if ld == cols:
        return torch.empty(rows, cols, dtype=dtype, device=device)
    return torch.empty(rows, ld, dtype=dtype, device=device)[:, :cols]


_STATS_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float8_e4m3fn)


def _update_forensic_role(tensor, role, mod):
    """Per-role statistics for forensic mode (apa/layers.py:63-106): max |x|,
    its first flat index, mean and standard deviation, computed on the device
    into the module's record for the role with no host synchronisation; the
    host reads the records only when a forensic snapshot needs them
    (APALinear._forensic_sync)."""
    if not mod.config.enable_forensic_logging:
        return
    with torch.no_grad():
        t = tensor.detach()
        if t.dtype not in _STATS_DTYPES:
            t = t.to(torch.float32)
        if not t.is_contiguous():
            t = t.contiguous()
        rec = mod._forensic_dev.get(role)
        if rec is None or rec.device != t.device:
            rec = torch.zeros(5, dtype=torch.int64, device=t.device)
            mod._forensic_dev[role] = rec
        _lib.check(_lib.lib().apa_tensor_stats(t.data_ptr(), _lib.dt_code(t.dtype), t.numel(), rec.data_ptr(),
                                               _lib.stream_handle(t.device)), "apa_tensor_stats")
        mod._forensic_last_shape[role] = list(tensor.shape)
        mod._forensic_pending.add(role)


class APABoundaryCast(nn.Module):
    """Casts activations to the parent layer's working dtype
    (apa/layers.py:10-21). Registered as a child so that module discovery and
    the manager's per-leaf telemetry buffers match the reference; APALinear's
    own forward fuses this cast into its kernels and does not call it."""

    def __init__(self, parent_linear):
        super().__init__()
        object.__setattr__(self, "parent_linear", parent_linear)

    def forward(self, x):
        wd = self.parent_linear.working_dtype
        if x.dtype == wd:
            return x
        return _BoundaryCastFn.apply(x, wd)


class _BoundaryCastFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wd):
        _lib.require_cuda(x, "APABoundaryCast")
        ctx.src_dtype = x.dtype
        x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        out = torch.empty(x2.shape, dtype=wd, device=x.device)
        st = _lib.lib().apa_cast(x2.data_ptr(), _lib.dt_code(x.dtype), x2.shape[0], x2.shape[1], x2.stride(0),
                                 out.data_ptr(), _lib.dt_code(wd), out.stride(0), None, 0, None, None, 0, None,
                                 None, _lib.stream_handle(x.device))
        _lib.check(st, "apa_cast")
        return out.view(x.shape)

    @staticmethod
    def backward(ctx, g):
        # ToCopyBackward: the gradient returns in the source dtype
        return g.to(ctx.src_dtype), None


# dgrad outputs of this step whose amax / NaN telemetry the dgrad kernel has
# already folded into the layer's boundary-cast buffers: data_ptr -> (weak
# reference to the dx tensor, boundary-cast module). A leaf module whose
# grad_output is one of these tensors (a LayerNorm or GELU feeding exactly one
# APALinear) merges that telemetry instead of reading the tensor again
# (manager.py:70-84 hooks). Cleared by APAManager.pre_step.
_DGRAD_TELEMETRY: dict = {}


def dgrad_telemetry_source(g):
    """The boundary-cast module whose buffers hold the telemetry of tensor g,
    when g is a live dgrad output of this step; else None."""
    e = _DGRAD_TELEMETRY.get(g.data_ptr())
    if e is None:
        return None
    t = e[0]()
    if t is None or t.data_ptr() != g.data_ptr() or t.shape != g.shape or t.dtype != g.dtype:
        return None
    return e[1]


class _APALinearFn(torch.autograd.Function):
    """Forward/backward of one APALinear on the fused kernels
    (apa/layers.py:109-303)."""

    @staticmethod
    def forward(ctx, x, weight_master, bias_master, mod):
        _lib.require_cuda(x, "APALinear")
        lib = _lib.lib()
        level = mod.level
        if mod._wq_level != level or mod._wq is None:
            mod._refresh(zero_pending=True)
        K, N = mod.in_features, mod.out_features
        if x.shape[-1] != K:
            raise RuntimeError(f"APALinear: input has {x.shape[-1]} features, expected {K}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, K)
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        M = x2.shape[0]
        wd = _working(level)
        dev = x.device
        s = _lib.stream_handle(dev)
        need_dx = ctx.needs_input_grad[0]
        need_dw = ctx.needs_input_grad[1]
        need_db = bias_master is not None and ctx.needs_input_grad[2]
        ydt = torch.float16 if level == LEVEL_FP16 else torch.float32
        f_on = mod.config.enable_forensic_logging
        if M == 0:
            ctx.empty = True
            ctx.lead, ctx.K, ctx.xdtype = lead, K, x.dtype
            return torch.empty(*lead, N, dtype=ydt, device=dev)
        ctx.empty = False

        # boundary cast (+ transposed copy for wgrad) with telemetry of x_cast
        # and the weight's pending amax (layers.py:17-21, :142-143)
        opc = _operand_code(level)
        if x.dtype == wd and level != LEVEL_TF32 and _tma_ok(x2):
            xq, new_xq = x2, False
        else:
            xq, new_xq = _alloc_2d(M, K, wd, dev), True
        xqt = _alloc_2d(K, M, wd, dev) if need_dw else None
        st = lib.apa_cast(x2.data_ptr(), _lib.dt_code(x.dtype), M, K, x2.stride(0),
                          xq.data_ptr() if new_xq else None, opc, xq.stride(0),
                          _lib.ptr(xqt), xqt.stride(0) if xqt is not None else 0,
                          mod.gpu_amax.data_ptr(), mod.gpu_has_nonfinite.data_ptr(), 0,
                          mod._w_pending.data_ptr(), None, s)
        _lib.check(st, "apa_cast(x)")

        y = torch.empty(M, N, dtype=ydt, device=dev)
        bq = mod._bq
        st = lib.apa_linear_fwd(level, xq.data_ptr(), xq.stride(0), mod._wq.data_ptr(), mod._wq.stride(0),
                                _lib.ptr(bq), y.data_ptr(), N, M, N, K, mod.gpu_amax.data_ptr(),
                                mod.gpu_has_nonfinite.data_ptr(), s)
        _lib.check(st, "apa_linear_fwd")

        if f_on:
            _update_forensic_role(xq, "input_activation", mod)
            _update_forensic_role(mod.weight_work, "weight", mod)
            _update_forensic_role(y, "output", mod)

        if need_dw or need_db:
            # a layer used several times in one step reports its gradients
            # ready (to the data-parallel buckets) after its last backward
            mod._bwd_pending += 1
        ctx.mod = mod
        ctx.level = level
        ctx.lead, ctx.M, ctx.N, ctx.K = lead, M, N, K
        ctx.xdtype = x.dtype
        ctx.xqt = xqt
        ctx.wqt = mod._wqt if need_dx else None
        ctx.flags = (need_dx, need_dw, need_db)
        return y.view(*lead, N)

    @staticmethod
    def backward(ctx, grad_output):
        if ctx.empty:
            need_dx = ctx.needs_input_grad[0]
            dx = torch.zeros(*ctx.lead, ctx.K, dtype=ctx.xdtype, device=grad_output.device) if need_dx else None
            return dx, None, None, None
        mod = ctx.mod
        lib = _lib.lib()
        level, M, N, K = ctx.level, ctx.M, ctx.N, ctx.K
        need_dx, need_dw, need_db = ctx.flags
        wd = _working(level)
        dev = grad_output.device
        s = _lib.stream_handle(dev)
        dy2 = grad_output.reshape(-1, N)
        if dy2.stride(-1) != 1:
            dy2 = dy2.contiguous()

        # grad_output telemetry (layers.py:211), its working-dtype copy, the
        # transposed copy for wgrad and the bias partial sums, in one pass
        if dy2.dtype == wd and level != LEVEL_TF32 and _tma_ok(dy2):
            dyq, new_dyq = dy2, False
        else:
            dyq, new_dyq = _alloc_2d(M, N, wd, dev), True
        dyqt = _alloc_2d(N, M, wd, dev) if need_dw else None
        nparts = (M + 63) // 64
        partial = torch.empty(nparts, N, dtype=torch.float32, device=dev) if need_db else None
        st = lib.apa_cast(dy2.data_ptr(), _lib.dt_code(dy2.dtype), M, N, dy2.stride(0),
                          dyq.data_ptr() if (new_dyq and need_dx) else None, _operand_code(level), dyq.stride(0),
                          _lib.ptr(dyqt), dyqt.stride(0) if dyqt is not None else 0,
                          mod.gpu_amax.data_ptr(), mod.gpu_has_nonfinite.data_ptr(), 1, None,
                          _lib.ptr(partial), s)
        _lib.check(st, "apa_cast(grad_output)")

        f_on = mod.config.enable_forensic_logging
        if f_on:
            _update_forensic_role(grad_output, "grad_output", mod)

        first = mod._grad_epoch != mod._epoch
        mod._grad_epoch = mod._epoch
        # weight and bias gradients first: in data-parallel runs their bucket
        # all-reduce then overlaps the input-gradient GEMM below
        dp = mod._dp
        if need_dw:
            W = mod.weight_master
            g = W.grad
            accumulate = 0 if (g is None or first) else 1
            if g is None:
                # data parallel: the bucket's view even when the caller cleared
                # the gradients after pre_step
                g = dp.grad_view(W) if dp is not None else None
                if g is None:
                    g = torch.empty_like(W)
            # scratch for the weight gradient: small gradients over long token
            # counts are split along the tokens (two kernels, fp32 partial sums),
            # and a last, partial wave of tiles is split along the tokens too
            # (stream-K: the splits' partials are added by the last to finish)
            nbytes = ctypes.c_int64(0)
            _lib.check(lib.apa_wgrad_workspace_bytes(level, M, N, K, ctypes.addressof(nbytes)),
                       "apa_wgrad_workspace_bytes")
            fused = dp.nvls_fused(mod, g) if (dp is not None and not accumulate) else None
            blocks = dp.weight_blocks(mod, g) if (dp is not None and not accumulate and fused is None) else None
            if fused is not None:
                # data parallel through NVLink SHARP: the GEMM's epilogue
                # averages the gradient's regions over the ranks as it goes
                ws = torch.empty(nbytes.value, dtype=torch.uint8, device=g.device) if nbytes.value > 0 else None
                st = lib.apa_linear_wgrad_dp(level, dyqt.data_ptr(), dyqt.stride(0), ctx.xqt.data_ptr(),
                                             ctx.xqt.stride(0), g.data_ptr(), K, M, N, K,
                                             mod._uf_counters.data_ptr(), mod.gpu_underflow_ratio.data_ptr(),
                                             _lib.ptr(ws), nbytes.value, *fused, s)
                _lib.check(st, "apa_linear_wgrad_dp")
                dp.nvls.queued(W)
            elif blocks:
                # data parallel: rows of the gradient in blocks, each block's
                # all-reduce issued as soon as its rows are written
                es = dyqt.element_size()
                for i, (r0, r1) in enumerate(blocks):
                    st = lib.apa_linear_wgrad_block(level, dyqt.data_ptr() + r0 * dyqt.stride(0) * es,
                                                    dyqt.stride(0), ctx.xqt.data_ptr(), ctx.xqt.stride(0),
                                                    g.data_ptr() + r0 * g.stride(0) * 4, g.stride(0), M, r1 - r0, K,
                                                    0, mod._uf_counters.data_ptr(),
                                                    mod.gpu_underflow_ratio.data_ptr(), int(i == len(blocks) - 1), s)
                    _lib.check(st, "apa_linear_wgrad_block")
                    dp.weight_block_done(mod, r0, r1)
            elif nbytes.value > 0:
                ws = torch.empty(nbytes.value, dtype=torch.uint8, device=g.device)
                st = lib.apa_linear_wgrad_ws(level, dyqt.data_ptr(), dyqt.stride(0), ctx.xqt.data_ptr(),
                                             ctx.xqt.stride(0), g.data_ptr(), K, M, N, K, accumulate,
                                             mod._uf_counters.data_ptr(), mod.gpu_underflow_ratio.data_ptr(),
                                             ws.data_ptr(), nbytes.value, s)
                _lib.check(st, "apa_linear_wgrad_ws")
            else:
                st = lib.apa_linear_wgrad(level, dyqt.data_ptr(), dyqt.stride(0), ctx.xqt.data_ptr(),
                                          ctx.xqt.stride(0), g.data_ptr(), K, M, N, K, accumulate,
                                          mod._uf_counters.data_ptr(), mod.gpu_underflow_ratio.data_ptr(), s)
                _lib.check(st, "apa_linear_wgrad")
            if W.grad is None:
                W.grad = g
            if f_on:
                _update_forensic_role(g, "grad_weight", mod)
        if need_db:
            b = mod.bias_master
            g = b.grad
            accumulate = 0 if (g is None or first) else 1
            if g is None:
                g = dp.grad_view(b) if dp is not None else None
                if g is None:
                    g = torch.empty_like(b)
            st = lib.apa_colsum_finalize(partial.data_ptr(), nparts, N, _lib.dt_code(wd), g.data_ptr(),
                                         accumulate, s)
            _lib.check(st, "apa_colsum_finalize")
            if b.grad is None:
                b.grad = g
        if need_dw or need_db:
            mod._bwd_pending -= 1
            if mod._bwd_pending <= 0:
                mod._notify_grad_ready()
        dx = None
        if need_dx:
            wqt = ctx.wqt
            if wqt is None or mod._wqt_stale:
                mod._make_wqt()
                wqt = mod._wqt
            dx = torch.empty(M, K, dtype=ctx.xdtype, device=dev)
            bc = mod.boundary_cast
            st = lib.apa_linear_dgrad(level, dyq.data_ptr(), dyq.stride(0), wqt.data_ptr(), wqt.stride(0),
                                      dx.data_ptr(), _lib.dt_code(ctx.xdtype), K, M, N, K,
                                      _lib.ptr(getattr(bc, "gpu_amax", None)),
                                      _lib.ptr(getattr(bc, "gpu_has_nonfinite", None)), s)
            _lib.check(st, "apa_linear_dgrad")
            dx = dx.view(*ctx.lead, K)
            # the kernel's telemetry is taken on the working-dtype values; dx
            # holds them exactly when it is fp32 or the working dtype itself
            if ctx.xdtype == torch.float32 or ctx.xdtype == mod.working_dtype:
                _DGRAD_TELEMETRY[dx.data_ptr()] = (weakref.ref(dx), bc)
        if f_on and dx is not None:
            _update_forensic_role(dx, "grad_input", mod)
        mod._needs_wt = need_dx
        ctx.xqt = None
        ctx.wqt = None
        return dx, None, None, None


def _drop_working_copy_keys(state_dict, prefix, *args):
    """The reference registers the working copies as parameters while a layer
    is at TF32 (its ``.to(float32)`` returns the master Parameter itself), so
    its checkpoints can carry ``weight_work`` / ``bias_work`` aliases of the
    masters. They are not state here; drop them so such checkpoints load."""
    for k in ("weight_work", "bias_work"):
        state_dict.pop(prefix + k, None)


class APALinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, config: APAConfig = APAConfig()):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.config = config
        dev = torch.device(config.device)
        # Parameters are initialised on the CPU generator and then moved, so a
        # given torch.manual_seed gives the same weights on every device.
        self.weight_master = nn.Parameter(torch.empty((out_features, in_features), dtype=torch.float32))
        if bias:
            self.bias_master = nn.Parameter(torch.empty(out_features, dtype=torch.float32))
        else:
            self.register_parameter("bias_master", None)
        self.weight_work = None
        self.bias_work = None
        self.level = LEVEL_FP8
        self.register_buffer("gpu_amax", torch.zeros(1, dtype=torch.float32, device=dev))
        self.register_buffer("gpu_underflow_ratio", torch.zeros(1, dtype=torch.float32, device=dev))
        self.register_buffer("gpu_has_nonfinite", torch.zeros(1, dtype=torch.int32, device=dev))
        # device scratch, not part of the state_dict: the weight's amax taken at
        # pre_step and merged at the next forward; the wgrad underflow counters
        self.register_buffer("_w_pending", torch.zeros(1, dtype=torch.float32, device=dev), persistent=False)
        self.register_buffer("_uf_counters", torch.zeros(3, dtype=torch.int64, device=dev), persistent=False)
        # weight amax of a working copy written by the fused optimizer step
        self.register_buffer("_w_pending_opt", torch.zeros(1, dtype=torch.float32, device=dev), persistent=False)
        self._prerefreshed = False     # the optimizer wrote the next working copy (APAAdamW)
        self._prerefresh_key = None
        self.ema_underflow_ratio = 0.0
        self.boundary_cast = APABoundaryCast(self)
        self._forensic_role_amax: dict = {}
        self._forensic_last_shape: dict = {}
        self._forensic_role_stats: dict = {}
        self._forensic_role_argmax: dict = {}
        self._forensic_dev: dict = {}          # role -> 5-word device record (apa_tensor_stats)
        self._forensic_pending: set = set()    # roles with device records newer than the dicts
        # working-copy buffers (recreated when the level changes)
        self._wq = None
        self._wqt = None
        self._bq = None
        self._wq_level = None
        self._wqt_stale = True
        self._needs_wt = True
        self._epoch = 0
        self._grad_epoch = -1
        self._grad_ready_cb = None
        self._dp = None                   # data-parallel gradient averager (buckets, row blocks)
        self._bwd_pending = 0             # forwards of this step whose weight/bias backward is still to run
        self._register_load_state_dict_pre_hook(_drop_working_copy_keys)
        self.reset_parameters()
        if dev.type != "cpu":
            with torch.no_grad():
                self.weight_master.data = self.weight_master.data.to(dev)
                if self.bias_master is not None:
                    self.bias_master.data = self.bias_master.data.to(dev)

    def reset_parameters(self) -> None:
        """Kaiming-uniform(a=sqrt(5)) weight and U(-1/sqrt(fan_in), 1/sqrt(fan_in))
        bias, as nn.Linear and the reference (apa/layers.py:353-358)."""
        nn.init.kaiming_uniform_(self.weight_master, a=math.sqrt(5))
        if self.bias_master is not None:
            fan_in = self.weight_master.shape[1]
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias_master, -bound, bound)

    @property
    def working_dtype(self):
        return _working(self.level)

    @property
    def current_threshold_min(self):
        return THRESHOLDS_MIN[self.level]

    # ------------------------------------------------------------------
    # working copies
    # ------------------------------------------------------------------
    def refresh_working_copy(self):
        """Cast the fp32 masters to the working dtype (apa/layers.py:368-372).
        At TF32 the working weight is the master itself, as in the reference."""
        self._refresh(zero_pending=True)

    def _refresh(self, zero_pending: bool) -> None:
        W = self.weight_master
        _lib.require_cuda(W, "APALinear.refresh_working_copy")
        lib = _lib.lib()
        s = _lib.stream_handle(W.device)
        level = self.level
        wd = _working(level)
        N, K = W.shape
        if zero_pending:
            self._w_pending.zero_()
        self._epoch += 1
        self._bwd_pending = 0
        with torch.no_grad():
            if level == LEVEL_TF32:
                # the working weight is the master itself (stored as a plain
                # attribute so it is not registered twice as a parameter); the
                # GEMM reads a TF32-rounded copy
                self.__dict__["weight_work"] = W
                if self._wq_level != level or self._wq is None or self._wq.dtype != wd:
                    self._wq = _alloc_2d(N, K, wd, W.device)
                new_wq = True
            else:
                if self._wq_level != level or self._wq is None or self._wq.dtype != wd:
                    self._wq = _alloc_2d(N, K, wd, W.device)
                self.weight_work = self._wq
                new_wq = True
            if self._wq_level != level or self._wqt is None or self._wqt.dtype != wd:
                self._wqt = _alloc_2d(K, N, wd, W.device)
            want_t = self._needs_wt
            if self._prerefreshed and self._prerefresh_key == (level, W._version, W.data_ptr()):
                # the fused optimizer step already wrote this working copy (and
                # its transpose if the backward wanted one) and its amax
                _lib.check(lib.apa_merge_telemetry(self._w_pending.data_ptr(), None,
                                                   self._w_pending_opt.data_ptr(), s), "apa_merge_telemetry")
                self._wqt_stale = not self._prerefresh_t
            else:
                st = lib.apa_cast(W.data_ptr(), _lib.DT_F32, N, K, W.stride(0),
                                  self._wq.data_ptr() if new_wq else None, _operand_code(level), self._wq.stride(0),
                                  self._wqt.data_ptr() if want_t else None, self._wqt.stride(0),
                                  self._w_pending.data_ptr(), None, 0, None, None, s)
                _lib.check(st, "apa_cast(weight)")
                self._wqt_stale = not want_t
            self._prerefreshed = False
            if self.bias_master is not None:
                b = self.bias_master
                if level == LEVEL_TF32:
                    self._bq = b.data
                    self.__dict__["bias_work"] = b
                else:
                    if self._bq is None or self._bq.dtype != wd or self._wq_level != level:
                        self._bq = torch.empty(N, dtype=wd, device=b.device)
                    st = lib.apa_cast(b.data_ptr(), _lib.DT_F32, 1, N, N, self._bq.data_ptr(), _lib.dt_code(wd), N,
                                      None, 0, None, None, 0, None, None, s)
                    _lib.check(st, "apa_cast(bias)")
                    self.bias_work = self._bq
        self._wq_level = level

    def _adamw_refresh(self, p, g, m, v, lr, beta1, beta2, eps, weight_decay, step) -> bool:
        """One AdamW step of weight_master fused with the next step's working
        copy (apa_adamw_cast): p, m, v updated in place, W_q (and W_q^T when
        the backward uses it) written at the current level, the weight amax
        kept for the next pre_step. False when the kernel cannot take this
        layout; the caller then updates p itself and pre_step casts as usual."""
        W = self.weight_master
        if p is not W or not (p.is_cuda and p.dim() == 2 and p.is_contiguous() and g.is_contiguous()
                              and g.dtype == torch.float32 and m.is_contiguous() and v.is_contiguous()):
            return False
        level = self.level
        wd = _working(level)
        N, K = W.shape
        if self._wq_level != level or self._wq is None or self._wq.dtype != wd:
            return False                  # buffers follow pre_step's allocation
        if self._wqt is None or self._wqt.dtype != wd:
            return False
        want_t = self._needs_wt
        s = _lib.stream_handle(W.device)
        lib = _lib.lib()
        st = lib.apa_adamw_cast(W.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), N, K, W.stride(0), lr, beta1,
                                beta2, eps, weight_decay, step, self._wq.data_ptr(), _operand_code(level),
                                self._wq.stride(0), self._wqt.data_ptr() if want_t else None, self._wqt.stride(0),
                                self._w_pending_opt.data_ptr(), s)
        if st == _lib.ERR_UNSUPPORTED:
            return False
        _lib.check(st, "apa_adamw_cast")
        self._prerefreshed = True
        self._prerefresh_key = (level, W._version, W.data_ptr())
        self._prerefresh_t = want_t
        return True

    def _make_wqt(self) -> None:
        """Transposed working weight for dgrad, made late when pre_step skipped it."""
        W = self.weight_master
        wd = _working(self.level)
        N, K = W.shape
        if self._wqt is None or self._wqt.dtype != wd:
            self._wqt = _alloc_2d(K, N, wd, W.device)
        st = _lib.lib().apa_cast(W.data_ptr(), _lib.DT_F32, N, K, W.stride(0), None, _operand_code(self.level), 0,
                                 self._wqt.data_ptr(), self._wqt.stride(0), None, None, 0, None, None,
                                 _lib.stream_handle(W.device))
        _lib.check(st, "apa_cast(weight^T)")
        self._wqt_stale = False

    def _notify_grad_ready(self):
        cb = self._grad_ready_cb
        if cb is not None:
            cb(self)

    # ------------------------------------------------------------------
    # telemetry entry points kept from the reference
    # ------------------------------------------------------------------
    def _forensic_sync(self):
        """Read the device records of the roles updated since the last read
        (one copy) into the per-role dictionaries the forensic snapshot uses:
        amax, and when configured mean/std (unbiased) and the argmax index."""
        if not self._forensic_pending:
            return
        c = self.config
        roles = sorted(self._forensic_pending)
        words = torch.stack([self._forensic_dev[r] for r in roles]).cpu().numpy().view(np.uint64)
        for role, w in zip(roles, words):
            key = int(w[0])
            amax = float(np.array([key >> 32], dtype=np.uint32).view(np.float32)[0])
            s1 = float(w[1:2].view(np.float64)[0])
            s2 = float(w[2:3].view(np.float64)[0])
            n = int(w[3])
            self._forensic_role_amax[role] = amax
            if c.forensic_capture_tensor_stats:
                mean = s1 / n if n else float("nan")
                std = math.sqrt(max((s2 - s1 * s1 / n) / (n - 1), 0.0)) if n > 1 and math.isfinite(s1) else (
                    float("nan") if n > 1 else 0.0)
                self._forensic_role_stats[role] = {"mean": mean, "std": std}
            if c.forensic_capture_argmax_index:
                self._forensic_role_argmax[role] = (~key) & 0xFFFFFFFF
        self._forensic_pending.clear()

    def track_telemetry(self, tensor: torch.Tensor, role: str = "unspecified"):
        """Running max of |tensor| into gpu_amax and the NaN/Inf flag
        (apa/layers.py:374-402); ``role`` matters only in forensic mode."""
        track_telemetry_on_tensor(tensor, self.gpu_amax, self.gpu_has_nonfinite)
        if self.config.enable_forensic_logging:
            _update_forensic_role(tensor, role, self)

    def update_underflow_metric(self, grad: torch.Tensor):
        """gpu_underflow_ratio = max(gpu_underflow_ratio, underflow ratio of grad)
        at this level's threshold (apa/layers.py:404-407)."""
        with torch.no_grad():
            update_running_underflow(grad, self.current_threshold_min, self.gpu_underflow_ratio)

    def forward(self, x):
        if self.weight_work is None or self._wq_level != self.level:
            self._refresh(zero_pending=True)
        return _APALinearFn.apply(x, self.weight_master, self.bias_master, self)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, " \
               f"bias={self.bias_master is not None}, level={self.level}"
