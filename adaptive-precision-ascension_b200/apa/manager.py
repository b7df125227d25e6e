"""APAManager: per-step lifecycle and the escalation ladder.

Same API as the reference (apa/manager.py:14-396): ``APAManager(model, config)``,
``pre_step()``, ``post_backward_sync_and_eval() -> bool``,
``get_trainable_parameters()``, plus the attributes its tests touch
(``apa_modules``, ``other_modules``, ``_escalate_module``,
``_forward_execution_order``, ``_forward_hook_handles``, ``forensic_logger``).

What changes underneath:

* pre_step zeroes every flag (and each layer's pending weight amax) with one
  launch, then refreshes each layer's working copy with one cast launch.
* post_backward_sync_and_eval runs the whole hard/soft evaluation as one
  device kernel (``apa_ladder_eval``) over all modules, then copies one small
  decision record to the host: one synchronisation per step, the same count
  as the reference's hard check (manager.py:189), instead of three ``.item()``
  per module on check steps. Levels and EMAs live on the device; the Python
  attributes ``module.level`` / ``module.ema_underflow_ratio`` stay
  authoritative (tests and users write them) and are re-uploaded whenever they
  differ from the last values the device reported.
* Data parallel (``torch.distributed`` initialised, world size > 1): the
  master gradients are averaged with NCCL all-reduces, started per bucket as
  soon as the backward has written them, and the per-module telemetry is
  combined with one int32 MAX all-reduce before the ladder kernel, so every
  rank skips the same batches and promotes the same layers (the reference
  evaluates only local values, manager.py:221-256).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from .config import APAConfig, LEVEL_FP8, LEVEL_FP16, LEVEL_TF32, THRESHOLDS_MAX
from .layers import APALinear
from .layers import dgrad_telemetry_source, _DGRAD_TELEMETRY
from .telemetry import APAEventLogger, APAForensicLogger, track_telemetry_on_tensor

_LEVEL_NAME = {LEVEL_FP8: "FP8", LEVEL_FP16: "FP16", LEVEL_TF32: "TF32"}
_KNOWN_ROLES = ("input_activation", "weight", "output", "grad_output", "grad_weight", "grad_input")
_REASONS = {1: "OVERFLOW", 2: "SILENT_UNDERFLOW"}


class _LadderState:
    """Device tables for the ladder kernel, rebuilt when a buffer moves."""

    def __init__(self, mgr: "APAManager", device, n_ready: int = 0):
        apa = list(mgr.apa_modules.values())
        oth = list(mgr.other_modules.values())
        self.L, self.O = len(apa), len(oth)
        self.key = mgr._buffer_key()
        i64 = dict(dtype=torch.int64, device=device)

        def table(ts):
            return torch.tensor([t.data_ptr() for t in ts] or [0], **i64)

        self.amax = table([m.gpu_amax for m in apa])
        self.ratio = table([m.gpu_underflow_ratio for m in apa])
        self.flag = table([m.gpu_has_nonfinite for m in apa])
        self.oamax = table([m.gpu_amax for m in oth])
        self.oflag = table([m.gpu_has_nonfinite for m in oth])
        self.zero = table([mgr._global_nonfinite] + [m.gpu_has_nonfinite for m in apa]
                          + [m.gpu_has_nonfinite for m in oth] + [m._w_pending for m in apa])
        self.nzero = 1 + 2 * self.L + self.O
        self.level = torch.zeros(max(self.L, 1), dtype=torch.int32, device=device)
        self.ema = torch.zeros(max(self.L, 1), dtype=torch.float64, device=device)
        self.host_level: Optional[List[int]] = None
        self.host_ema: Optional[List[float]] = None
        # data parallel: the packed telemetry the ranks MAX-reduce, followed by
        # the gradient averager's ready mask (one word per averaged parameter)
        self.n_ready = n_ready
        self.ready_off = 1 + 3 * self.L + 2 * self.O
        self.packed = torch.zeros(self.ready_off + n_ready, dtype=torch.int32, device=device)
        self.ready_host = torch.zeros(max(1, n_ready), dtype=torch.int32, pin_memory=device.type == "cuda")
        nint = 4 + 2 * self.L + self.O
        self.dbl_off = (nint * 4 + 7) & ~7
        self.nbytes = self.dbl_off + 8 * (2 * self.L + self.O)
        self.out = torch.zeros(self.nbytes, dtype=torch.uint8, device=device)
        self.out_host = torch.zeros(self.nbytes, dtype=torch.uint8, pin_memory=True)

    def parse(self):
        raw = self.out_host.numpy()
        L, O = self.L, self.O
        ints = raw[: (4 + 2 * L + O) * 4].view(np.int32)
        dbl = raw[self.dbl_off: self.dbl_off + 8 * (2 * L + O)].view(np.float64)
        return dict(status=int(ints[0]), min_level=int(ints[1]), code=ints[4:4 + L], ocode=ints[4 + L:4 + L + O],
                    level=ints[4 + L + O:4 + 2 * L + O], ema=dbl[:L], trig=dbl[L:2 * L], otrig=dbl[2 * L:])


class APAManager:
    def __init__(self, model: nn.Module, config: APAConfig = APAConfig(), process_group=None,
                 sync_gradients: bool = True, bucket_bytes: int = 64 << 20, dp_reserved_sms: int = 16,
                 dp_max_ctas: int = 0, dp_block_bytes: int = 0, dp_block_rows: int = 0, dp_nvls: bool = False):
        self.model = model
        self.config = config
        self.step_count = 0
        self.apa_modules: Dict[str, APALinear] = {}
        self.other_modules: Dict[str, nn.Module] = {}
        self._global_nonfinite = torch.zeros(1, dtype=torch.int32, device=config.device)
        self.logger = APAEventLogger(config.log_file)
        self.forensic_logger: Optional[APAForensicLogger] = None
        self._forward_execution_order: List[str] = []
        self._forward_hook_handles = []
        self._register_modules_and_hooks()
        if config.enable_forensic_logging:
            self.forensic_logger = APAForensicLogger(config.forensic_log_file)
            self._register_forensic_forward_hooks()
        self._ladder: Optional[_LadderState] = None
        self._pg = process_group
        self._telem_pg = None          # second communicator for the small telemetry reduction
        self._sync_gradients = sync_gradients
        self._bucket_bytes = bucket_bytes
        self._dp_reserved_sms = dp_reserved_sms   # SMs the GEMMs leave free while a reduction runs
        self._dp_max_ctas = dp_max_ctas           # >0: gradient communicator capped at this many CTAs
        self._dp_block_bytes = dp_block_bytes     # weights this large are reduced in row blocks (0: never)
        self._dp_block_rows = dp_block_rows       # rows per block (0: one GEMM wave)
        self._dp_nvls = dp_nvls                   # opt-in: large weight gradients averaged through NVLink SHARP
        self._dp = None

    # ------------------------------------------------------------------
    # discovery (manager.py:70-109)
    # ------------------------------------------------------------------
    def _register_modules_and_hooks(self):
        for name, module in self.model.named_modules():
            if isinstance(module, APALinear):
                self.apa_modules[name] = module
            elif len(list(module.children())) == 0:
                self.other_modules[name] = module
                dev = self.config.device
                module.register_buffer("gpu_amax", torch.zeros(1, dtype=torch.float32, device=dev), persistent=False)
                module.register_buffer("gpu_has_nonfinite", torch.zeros(1, dtype=torch.int32, device=dev),
                                       persistent=False)

                def hook_fn(mod, grad_input, grad_output):
                    for g in grad_output:
                        if g is None:
                            continue
                        src = dgrad_telemetry_source(g) if g.is_cuda else None
                        if src is not None:
                            # g is an APALinear's dgrad output whose telemetry is
                            # already in its boundary-cast buffers: both modules'
                            # buffers see the same values and are reset together
                            _lib.check(_lib.lib().apa_merge_telemetry(mod.gpu_amax.data_ptr(),
                                                                      mod.gpu_has_nonfinite.data_ptr(),
                                                                      src.gpu_amax.data_ptr(),
                                                                      _lib.stream_handle(g.device)),
                                       "apa_merge_telemetry")
                        else:
                            track_telemetry_on_tensor(g, mod.gpu_amax, mod.gpu_has_nonfinite)

                # APALinear fuses its boundary cast into its kernels (the cast
                # module is never called), and its dgrad kernel writes this
                # hook's telemetry into the cast module's buffers directly.
                module.register_full_backward_hook(hook_fn)

    def _register_forensic_forward_hooks(self):
        for name, module in self.apa_modules.items():
            def make_hook(module_name):
                def _fwd_hook(mod, inp, out):
                    self._forward_execution_order.append(module_name)
                return _fwd_hook
            self._forward_hook_handles.append(module.register_forward_hook(make_hook(name)))

    # ------------------------------------------------------------------
    # parameter registry (manager.py:115-139)
    # ------------------------------------------------------------------
    def get_trainable_parameters(self) -> List[nn.Parameter]:
        params, seen = [], set()
        for module in self.apa_modules.values():
            for p in (module.weight_master, module.bias_master):
                if p is not None and p.requires_grad and id(p) not in seen:
                    params.append(p)
                    seen.add(id(p))
        for p in self.model.parameters():
            if p.requires_grad and id(p) not in seen:
                params.append(p)
                seen.add(id(p))
        expected = sum(1 for p in self.model.parameters() if p.requires_grad)
        assert len(params) == expected, f"Parameter count mismatch: found {len(params)}, expected {expected}"
        return params

    # ------------------------------------------------------------------
    # device tables
    # ------------------------------------------------------------------
    def _buffer_key(self):
        k = [self._global_nonfinite.data_ptr()]
        for m in self.apa_modules.values():
            k += [m.gpu_amax.data_ptr(), m.gpu_underflow_ratio.data_ptr(), m.gpu_has_nonfinite.data_ptr(),
                  m._w_pending.data_ptr()]
        for m in self.other_modules.values():
            k += [m.gpu_amax.data_ptr(), m.gpu_has_nonfinite.data_ptr()]
        return tuple(k)

    def _state(self) -> _LadderState:
        st = self._ladder
        n_ready = len(self._dp.order) if self._dp is not None else 0
        if st is None or st.key != self._buffer_key() or st.n_ready != n_ready:
            self._ladder = st = _LadderState(self, self._global_nonfinite.device, n_ready)
        return st

    # ------------------------------------------------------------------
    # per-step lifecycle
    # ------------------------------------------------------------------
    def pre_step(self):
        """Zero the per-step flags (not amax: it persists across the check
        window) and refresh every working copy (manager.py:145-172)."""
        _DGRAD_TELEMETRY.clear()
        st = self._state()
        s = _lib.stream_handle(self._global_nonfinite.device)
        _lib.check(_lib.lib().apa_zero_list(st.zero.data_ptr(), st.nzero, s), "apa_zero_list")
        for module in self.apa_modules.values():
            module._refresh(zero_pending=False)
        if self._sync_gradients and self._world() > 1:
            self._averager().arm()
        if self.config.enable_forensic_logging:
            self._forward_execution_order.clear()
            for module in self.apa_modules.values():
                module._forensic_role_amax.clear()
                module._forensic_pending.clear()

    def _sync_grads_to_master(self):
        """The weight-gradient kernels write the fp32 master gradients directly
        (manager.py:191-204 becomes a no-op on the fused path). A gradient that
        reached a working copy some other way is still copied over."""
        with torch.no_grad():
            for module in self.apa_modules.values():
                for work, master in ((module.weight_work, module.weight_master),
                                     (module.bias_work, module.bias_master)):
                    if work is None or master is None or work is master or work.grad is None:
                        continue
                    g = work.grad.to(torch.float32)
                    if master.grad is None:
                        master.grad = g.clone()
                    else:
                        master.grad.copy_(g)

    def _dist(self):
        if not torch.distributed.is_available() or not torch.distributed.is_initialized():
            return None
        return self._pg

    def _world(self) -> int:
        if not torch.distributed.is_available() or not torch.distributed.is_initialized():
            return 1
        return torch.distributed.get_world_size(self._pg)

    def _upload_ladder(self, st: _LadderState):
        levels = [int(m.level) for m in self.apa_modules.values()]
        emas = [float(m.ema_underflow_ratio) for m in self.apa_modules.values()]
        if levels != st.host_level or emas != st.host_ema:
            if st.L:
                st.level[: st.L].copy_(torch.tensor(levels, dtype=torch.int32))
                st.ema[: st.L].copy_(torch.tensor(emas, dtype=torch.float64))
            st.host_level, st.host_ema = levels, emas

    def _telemetry_group(self):
        """The telemetry MAX reduction runs on its own communicator so it does
        not queue behind the gradient buckets still in flight on the main one
        (collectives of one communicator run in issue order)."""
        if self._telem_pg is None:
            dist = torch.distributed
            ranks = dist.get_process_group_ranks(self._pg) if self._pg is not None else list(
                range(dist.get_world_size()))
            self._telem_pg = dist.new_group(ranks=ranks, use_local_synchronization=True)
        return self._telem_pg

    def _run_ladder(self, before_wait=None) -> dict:
        """One ladder evaluation. before_wait() (if given) is called once the
        decision record's device-to-host copy is queued and before the host
        waits for it: work it queues on the stream does not delay the record."""
        st = self._state()
        self._upload_ladder(st)
        lib = _lib.lib()
        dev = self._global_nonfinite.device
        s = _lib.stream_handle(dev)
        glob = None
        if self._world() > 1:
            _lib.check(lib.apa_ladder_pack(st.L, st.amax.data_ptr(), st.ratio.data_ptr(), st.flag.data_ptr(), st.O,
                                           st.oamax.data_ptr(), st.oflag.data_ptr(), st.packed.data_ptr(), s),
                       "apa_ladder_pack")
            if st.n_ready:
                st.packed[st.ready_off:].copy_(self._dp.ready_mask(), non_blocking=True)
            torch.distributed.all_reduce(st.packed, op=torch.distributed.ReduceOp.MAX, group=self._telemetry_group())
            if st.n_ready:
                # read back with the decision record (same stream, same host wait)
                st.ready_host[: st.n_ready].copy_(st.packed[st.ready_off:], non_blocking=True)
            glob = st.packed.data_ptr()
        _lib.check(lib.apa_ladder_eval(st.L, st.amax.data_ptr(), st.ratio.data_ptr(), st.flag.data_ptr(),
                                       st.level.data_ptr(), st.ema.data_ptr(), st.O, st.oamax.data_ptr(),
                                       st.oflag.data_ptr(), glob, self.step_count, self.config.check_interval,
                                       float(self.config.theta_underflow), float(self.config.ema_alpha),
                                       st.out.data_ptr(), st.out_host.data_ptr(), s), "apa_ladder_eval")
        if before_wait is None:
            torch.cuda.current_stream(dev).synchronize()
        else:
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(dev))
            before_wait()
            done.synchronize()
        rec = st.parse()
        if rec["status"] & 0x100:
            bits = _lib.device_status(clear=True)
            raise _lib.APAKernelError(
                f"a kernel's bounded wait gave up (device status 0x{bits:x}): a stalled pipeline, or in data "
                "parallel runs a rank that did not reach the same reduction")
        if rec["status"] & 1:
            lv = [int(v) for v in rec["level"]]
            em = [float(v) for v in rec["ema"]]
            for m, l, e in zip(self.apa_modules.values(), lv, em):
                m.level = l
                m.ema_underflow_ratio = e
            st.host_level, st.host_ema = lv, em
        return rec

    def _check_hard_overflow(self) -> bool:
        """OR of every module's NaN/Inf flag (manager.py:178-189)."""
        with torch.no_grad():
            self._global_nonfinite.zero_()
            flags = [m.gpu_has_nonfinite for m in self.apa_modules.values()]
            flags += [m.gpu_has_nonfinite for m in self.other_modules.values()]
            for f in flags:
                torch.maximum(self._global_nonfinite, (f > 0).to(torch.int32), out=self._global_nonfinite)
            if self._world() > 1:
                torch.distributed.all_reduce(self._global_nonfinite, op=torch.distributed.ReduceOp.MAX,
                                             group=self._pg)
            return self._global_nonfinite.item() > 0

    def _do_full_evaluation(self) -> bool:
        """One soft evaluation regardless of the step counter (manager.py:206-261)."""
        saved = self.config.check_interval
        try:
            self.config.check_interval = 1
            rec = self._run_ladder()
        finally:
            self.config.check_interval = saved
        self._log_record(rec)
        return not (rec["status"] & 2)

    # ------------------------------------------------------------------
    # escalation (manager.py:267-381)
    # ------------------------------------------------------------------
    def _escalate_module(self, name: str, module: APALinear, reason: str, trigger_value: float):
        """Host-side escalation, as the reference's: one level up (capped at
        TF32), EMA reset, event logged. The next ladder launch picks up the
        new level from the module attribute."""
        old_level = module.level
        if old_level < LEVEL_TF32:
            module.level += 1
            module.ema_underflow_ratio = 0.0
            self._log_escalation(name, module, reason, old_level, trigger_value)

    def _log_escalation(self, name, module, reason, old_level, trigger_value):
        self.logger.log_escalation(self.step_count, name, reason, old_level, module.level, trigger_value)
        if self.config.enable_forensic_logging and self.forensic_logger is not None:
            self._capture_forensic_snapshot(name, module, reason, old_level, trigger_value)

    def _capture_forensic_snapshot(self, name, module, reason, old_level, trigger_value):
        module._forensic_sync()
        role_amax = dict(module._forensic_role_amax)
        culprit_role, culprit_amax = None, -1.0
        for role, val in role_amax.items():
            if val > culprit_amax:
                culprit_amax, culprit_role = val, role
        per_role_stats = None
        if self.config.forensic_capture_tensor_stats and module._forensic_role_stats:
            per_role_stats = {r: module._forensic_role_stats.get(r) for r in _KNOWN_ROLES}
        argmax_index = None
        if self.config.forensic_capture_argmax_index and culprit_role:
            argmax_index = module._forensic_role_argmax.get(culprit_role)
        preceding = None
        if name in self._forward_execution_order:
            idx = self._forward_execution_order.index(name)
            if idx > 0:
                preceding = self._forward_execution_order[idx - 1]
        dtype_str = {LEVEL_FP8: "float8_e4m3fn", LEVEL_FP16: "float16", LEVEL_TF32: "float32"}
        record = {
            "step": self.step_count,
            "module_name": name,
            "reason": reason,
            "level_before": _LEVEL_NAME.get(old_level, str(old_level)),
            "level_after": _LEVEL_NAME.get(module.level, str(module.level)),
            "culprit_tensor_role": culprit_role,
            "per_role_amax": {r: role_amax.get(r) for r in _KNOWN_ROLES},
            "amax_value": float(trigger_value),
            "threshold_at_time": THRESHOLDS_MAX.get(old_level, float("inf")),
            "tensor_shape": module._forensic_last_shape.get(culprit_role) if culprit_role else None,
            "dtype_at_time": dtype_str.get(old_level, "unknown"),
            "preceding_module_in_forward_order": preceding,
            "underflow_ratio": module.ema_underflow_ratio if reason == "SILENT_UNDERFLOW" else None,
            "argmax_flat_index": argmax_index,
            "per_role_stats": per_role_stats,
        }
        self.forensic_logger.log_forensic_event(record)

    def _log_record(self, rec: dict):
        """Emit the reference's events for one ladder decision record
        (manager.py:221-259), in its order."""
        if not (rec["status"] & 1):
            return
        names = list(self.apa_modules.keys())
        mods = list(self.apa_modules.values())
        triggers = []
        for i, c in enumerate(rec["code"]):
            c = int(c)
            reason = c & 3
            if not reason:
                continue
            if reason == 1:
                triggers.append(names[i])
            if c & 4:
                old = (c >> 4) & 3
                self._log_escalation(names[i], mods[i], _REASONS[reason], old, float(rec["trig"][i]))
        min_level = rec["min_level"]
        for j, (oname, oc) in enumerate(zip(self.other_modules.keys(), rec["ocode"])):
            if oc:
                triggers.append(oname)
                self.logger.log_escalation(self.step_count, oname, "NON_PARAMETRIC_OVERFLOW", min_level, min_level,
                                           float(rec["otrig"][j]))
        if rec["status"] & 2:
            self.logger.log_skip_batch(self.step_count, "OVERFLOW_DETECTED", triggers)

    # ------------------------------------------------------------------
    # main entry point (manager.py:387-396)
    # ------------------------------------------------------------------
    def post_backward_sync_and_eval(self) -> bool:
        self.step_count += 1
        self._sync_grads_to_master()
        join = None
        if self._sync_gradients and self._world() > 1:
            # the remaining gradient buckets go out now; the stream joins them
            # after the ladder's record copy, so the decision does not wait
            # for the bulk reduction (the optimizer step, queued later, does)
            avg = self._averager()
            avg.issue_remaining()
            join = avg.finish
        rec = self._run_ladder(before_wait=join)
        st = self._ladder
        if join is not None and st is not None and st.n_ready:
            # parameters no rank produced a gradient for: grad None, as on one GPU
            self._dp.drop_unused(st.ready_host[: st.n_ready])
        self._log_record(rec)
        return not (rec["status"] & 2)

    def no_sync(self):
        """Context for gradient accumulation under data parallelism: backward
        passes inside it accumulate into the gradient buckets without reducing
        them; the step's last backward runs outside it and starts the
        reductions (a no-op context on one process)."""
        import contextlib
        if self._sync_gradients and self._world() > 1:
            return self._averager().no_sync()
        return contextlib.nullcontext()

    # ------------------------------------------------------------------
    # data parallel gradients
    # ------------------------------------------------------------------
    def _averager(self):
        from .dp import GradientAverager
        if self._dp is None:
            self._dp = GradientAverager(self, self._pg, self._bucket_bytes, self._dp_reserved_sms,
                                        self._dp_max_ctas, self._dp_block_bytes, self._dp_block_rows,
                                        nvls=self._dp_nvls)
        return self._dp

    def _allreduce_grads(self):
        self._averager().finish()
