"""Data-parallel gradient averaging for APAManager.

The reference has no gradient synchronisation at all (its only collective is
the overflow flag, manager.py:186-187). Data parallel training here averages
every trainable gradient across ranks once per step. Gradients are grouped
into flat buckets (in reverse registration order, roughly the order the
backward produces them; 64 MiB each by default: on two GPUs the char-level
GPT ran at 6.89 ms per step with them against 7.07 ms with 5.5 MiB buckets,
because the GEMMs leave SMs to the collective from the first bucket on).
Each parameter's ``.grad`` is a view into its bucket, so the weight-gradient
kernels and autograd write straight into the buffers that NCCL reduces, with
no packing copies. A bucket's all-reduce is
issued (asynchronously, on the process group's stream) as soon as all of its
gradients are written, and buckets are issued in a fixed order so every rank
runs the same collectives in the same sequence.

Optionally (``block_bytes`` > 0; off by default) large APALinear weights sit
alone in their bucket and are reduced in row blocks: the layer's backward
computes the weight gradient one block of output rows at a time
(``apa_linear_wgrad_block``) and the block's all-reduce starts as soon as its
rows are written, while the next block and the input-gradient GEMM run. A
block holds as many 256-row tile rows as one wave of the GEMMs (on the SMs
left beside the collective) covers. Results are bit-identical to the
whole-bucket reduction; on two B200s the single-layer 8192x4096x4096 step was
slower with blocks (0.60-0.66 ms against 0.56 ms for 1024- and 2048-row
blocks, with and without SM reserves or a CTA-capped communicator), so the
whole-bucket reduction overlapping the input-gradient GEMM stays the default.

Every trainable floating-point parameter is averaged: parameters of another
dtype than fp32 (a bf16 LayerNorm, an fp16 embedding) get buckets of their
own dtype. A gradient that autograd produced outside its bucket (the caller
cleared it after ``pre_step``) is copied into the bucket view by the
parameter's post-accumulate hook, so every rank reduces the same buffers with
the same collectives. Gradient accumulation over several backward passes in
one step: all but the last run inside ``no_sync()``; a second backward of the
same parameters outside it raises, since its buckets are already reduced.
Parameters that received no gradient on any rank in a step end it with
``grad = None`` (as on one GPU, so the optimizer skips them): which
parameters were ready travels as a mask in the manager's per-step telemetry
all-reduce (``ready_mask`` / ``drop_unused``), or in its own small
all-reduce (``sync_unused``) for callers without the manager.

Optionally (``nvls=True``, ``APAManager(dp_nvls=True)``; off by default),
APALinear weights of 1 Mi elements or more skip the NCCL buckets when the
GPUs support NVLink multicast: their gradients are averaged through NVLink
SHARP by the library's own kernels (``_NvlsGradients``), each as soon as its
weight-gradient GEMM has written it. On two B200s it measured level with the
NCCL buckets (the single 8192x4096x4096 layer 0.575 against 0.557 ms per
step, GPT-2-medium 387 K against 382 K tokens/s); NCCL itself reduces through
NVLS on NVSwitch systems, so the buckets stay the default.
"""
from __future__ import annotations

import contextlib
import ctypes
from typing import Dict, List

import torch
import torch.distributed as dist


class _Bucket:
    def __init__(self, params: List[torch.nn.Parameter], device):
        self.params = params
        self.dtype = params[0].dtype
        self.numel = sum(p.numel() for p in params)
        self.flat = torch.zeros(self.numel, dtype=self.dtype, device=device)
        self.views: Dict[int, torch.Tensor] = {}
        off = 0
        for p in params:
            self.views[id(p)] = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()
        self.pending = len(params)
        self.handles = []
        self.blocks = None            # row blocks of a single large weight, reduced as they finish
        self.blocks_issued = False


# SMs left to the collective's kernel while a bucket all-reduce is in flight:
# the persistent GEMMs otherwise occupy every SM and the all-reduce could only
# start after them.
RESERVED_SMS = 16


def _capped_nccl_group(process_group, max_ctas: int):
    """A second NCCL communicator over the same ranks whose kernels use at most
    max_ctas CTAs: a long backward can then carry the reductions on a few SMs
    instead of losing a large share of every SM-wide kernel to them."""
    ranks = dist.get_process_group_ranks(process_group) if process_group is not None else list(
        range(dist.get_world_size()))
    opts = dist.ProcessGroupNCCL.Options()
    opts.config.max_ctas = max_ctas
    opts.config.min_ctas = 1
    opts.config.nvls_ctas = max_ctas
    return dist.new_group(ranks=ranks, backend="nccl", pg_options=opts, use_local_synchronization=True)


class _NvlsGradients:
    """APALinear weight gradients averaged through NVLink SHARP instead of
    NCCL: the fp32 gradients of the chosen weights live in one symmetric
    allocation bound to an NVLink multicast object (each weight's `.grad` is a
    view into it, so the weight-gradient kernel writes there), cut into
    regions of 32 rows x 64 columns, each averaged over the ranks by one
    owner rank (multimem.ld_reduce through the switch, multimem.st of the
    mean to every rank). The weight-gradient GEMM does it in its epilogue
    (apa_linear_wgrad_dp: every region published as soon as it is stored,
    the owned ones averaged while the tensor cores compute later tiles; a
    gradient the plan splits along the tokens leaves its owned regions to
    apa_dp_region_reduce on a side stream); gradients written otherwise take
    the standalone kernels (apa_dp_region_signal, then apa_dp_region_reduce
    on the side stream). A one-thread apa_dp_region_wait on the side stream
    marks the gradient complete; the step's later work joins that stream. Per GPU and gradient
    of B bytes about B crosses NVLink each way whatever the number of ranks,
    against 2 (world - 1) / world B for a ring all-reduce.

    Every rank must produce and reduce these gradients in every step: a rank
    that did not run one of these layers raises at the end of its backward
    (GradientAverager.issue_remaining); a rank that skips the step altogether
    makes the others' bounded waits expire, which the next ladder decision
    reports as an error."""

    def __init__(self, params, pg, world: int, rank: int, device, ctas: int):
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        lib = _lib.lib()
        self.world, self.rank, self.ctas = world, rank, ctas
        self.index: Dict[int, int] = {}
        self.offset: Dict[int, int] = {}
        self.regions: Dict[int, int] = {}
        off = 0
        for i, p in enumerate(params):
            self.index[id(p)] = i
            self.offset[id(p)] = off
            off += (p.numel() + 63) // 64 * 64          # 256-byte aligned gradients
            n = ctypes.c_int64(0)
            _lib.check(lib.apa_dp_regions(p.shape[0], p.shape[1], ctypes.addressof(n)), "apa_dp_regions")
            self.regions[id(p)] = n.value
        # counters (u32 words) per gradient: done, epoch, 2 spare, then one
        # ready word per region and one deferred word per region, each run
        # rounded up to 16 bytes
        self.ctr: Dict[int, int] = {}
        for p in params:
            self.ctr[id(p)] = off
            off += 4 + 2 * ((self.regions[id(p)] + 3) // 4 * 4)
        idx = device.index if device.index is not None else torch.cuda.current_device()
        if not symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, idx):
            raise RuntimeError("no NVLink multicast support")
        buf = symm.empty(off, dtype=torch.float32, device=device)
        group = pg if pg is not None else dist.group.WORLD
        hdl = symm.rendezvous(buf, group)
        if not int(hdl.multicast_ptr):
            raise RuntimeError("no multicast mapping for the gradient buffer")
        base_local = int(hdl.buffer_ptrs[hdl.rank])
        self.mc = int(hdl.multicast_ptr) + (buf.data_ptr() - base_local)
        self.buf, self.hdl = buf, hdl
        buf.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self.views = {id(p): buf[self.offset[id(p)]:self.offset[id(p)] + p.numel()].view_as(p) for p in params}
        self.params = list(params)
        self.stream = None
        self.pending = False
        self.fused_now = set()          # reduced by their weight-gradient GEMM this step
        self.fused_calls = 0            # gradients reduced by their GEMM / by the standalone kernels
        self.standalone_calls = 0

    def _word(self, p, word: int, multicast: bool) -> int:
        byte = (self.ctr[id(p)] + word) * 4
        return (self.mc if multicast else self.buf.data_ptr()) + byte

    def _counters(self, p):
        """(ready local, ready multicast, done multicast, epoch local,
        deferred local)."""
        deferred = 4 + (self.regions[id(p)] + 3) // 4 * 4
        return (self._word(p, 4, False), self._word(p, 4, True), self._word(p, 0, True), self._word(p, 1, False),
                self._word(p, deferred, False))

    def fused_args(self, p):
        """The data-parallel arguments of apa_linear_wgrad_dp for p's
        gradient (its view in this buffer): multicast address, counters,
        world, rank. The caller launches the GEMM, then calls queued(p)."""
        return (self.mc + self.offset[id(p)] * 4, *self._counters(p), self.world, self.rank)

    def _side(self):
        dev = self.buf.device
        if self.stream is None:
            self.stream = torch.cuda.Stream(device=dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        return self.stream.cuda_stream

    def _wait(self, p, sh) -> None:
        from . import _lib
        _lib.check(_lib.lib().apa_dp_region_wait(self._word(p, 0, False), self._word(p, 1, False),
                                                 self.regions[id(p)], sh), "apa_dp_region_wait")
        self.pending = True

    def queued(self, p) -> None:
        """p's weight-gradient GEMM (apa_linear_wgrad_dp) is queued on the
        current stream: the regions it left to the side stream (split
        gradients), then the completion wait, go on the side stream."""
        from . import _lib
        self.fused_now.add(id(p))
        self.fused_calls += 1
        sh = self._side()
        rows, cols = p.shape
        _lib.check(_lib.lib().apa_dp_region_reduce(self.mc + self.offset[id(p)] * 4, cols, rows, cols,
                                                   *self._counters(p), self.world, self.rank, 1, 4, sh),
                   "apa_dp_region_reduce")
        self._wait(p, sh)

    def reduce(self, p) -> None:
        """Average p's gradient over the ranks (queued; see join). A gradient
        its GEMM already reduces needs nothing more."""
        if id(p) in self.fused_now:
            return
        from . import _lib
        lib = _lib.lib()
        dev = self.buf.device
        rows, cols = p.shape
        ctr = self._counters(p)
        mc = self.mc + self.offset[id(p)] * 4
        _lib.check(lib.apa_dp_region_signal(mc, cols, rows, cols, *ctr, self.world, self.rank,
                                            _lib.stream_handle(dev)), "apa_dp_region_signal")
        sh = self._side()
        _lib.check(lib.apa_dp_region_reduce(mc, cols, rows, cols, *ctr, self.world, self.rank, 0, self.ctas, sh),
                   "apa_dp_region_reduce")
        self.standalone_calls += 1
        self._wait(p, sh)

    def step_begin(self) -> None:
        self.fused_now.clear()

    def join(self, stream) -> None:
        if self.pending:
            stream.wait_stream(self.stream)
            self.pending = False


def _nvls_candidates(mgr, min_elems: int):
    out = []
    for m in mgr.apa_modules.values():
        W = m.weight_master
        if W.requires_grad and W.is_cuda and W.dtype == torch.float32 and W.numel() >= min_elems and \
                W.dim() == 2 and W.shape[1] % 4 == 0:
            out.append(W)
    return out


class GradientAverager:
    def __init__(self, mgr, process_group=None, bucket_bytes: int = 64 << 20, reserved_sms: int = RESERVED_SMS,
                 max_ctas: int = 0, block_bytes: int = 0, block_rows: int = 0, nvls: bool = False,
                 nvls_min_elems: int = 1 << 20):
        self.world = dist.get_world_size(process_group)
        if max_ctas > 0 and dist.get_backend(process_group) == "nccl":
            process_group = _capped_nccl_group(process_group, max_ctas)
            reserved_sms = max_ctas
        self.pg = process_group
        self.reserved_sms = reserved_sms
        self.avg_op = dist.ReduceOp.AVG if dist.get_backend(process_group) == "nccl" else None
        # buckets follow the order in which backward produces gradients, which
        # is close to the reverse of registration (module definition) order;
        # buckets are issued strictly in order, so one bucket holding an early
        # layer's gradient would hold back every bucket after it
        trainable = {id(p) for p in mgr.get_trainable_parameters() if p.is_floating_point()}
        params, seen = [], set()
        for p in mgr.model.parameters():
            if id(p) in trainable and id(p) not in seen:
                params.append(p)
                seen.add(id(p))
        params = list(reversed(params))
        device = params[0].device if params else torch.device("cpu")
        # large APALinear weight gradients through NVLink SHARP when the
        # communicator is NCCL on GPUs with NVLink multicast; the rest (and
        # everything when that is unavailable) in NCCL buckets
        self.nvls = None
        if nvls and device.type == "cuda" and dist.get_backend(process_group) == "nccl" and self.world > 1:
            cands = [p for p in _nvls_candidates(mgr, nvls_min_elems) if id(p) in trainable]
            if cands:
                try:
                    self.nvls = _NvlsGradients(cands, process_group, self.world,
                                               dist.get_rank(process_group), device, max(1, reserved_sms))
                except Exception as e:   # no symmetric memory / multicast here: NCCL for everything
                    import warnings
                    warnings.warn(f"NVLS gradient averaging unavailable ({e!r}); using NCCL buckets")
                    self.nvls = None
        if self.nvls is not None:
            params = [p for p in params if id(p) not in self.nvls.index]
        self.bucket_bytes = bucket_bytes
        owner = {id(m.weight_master): m for m in mgr.apa_modules.values()}
        blocked = {}
        if block_bytes > 0:
            for p in params:
                m = owner.get(id(p))
                if m is not None and p.dim() == 2 and p.numel() * 4 >= block_bytes:
                    blocks = self._row_blocks(p, reserved_sms, block_rows)
                    if len(blocks) >= 2:
                        blocked[id(p)] = (m, blocks)
        # one bucket in the making per dtype (a bucket is one flat tensor of one
        # dtype); flushed when full, before a row-blocked weight, and at the
        # end in the order the dtypes first appeared
        self.buckets: List[_Bucket] = []
        cur: Dict[torch.dtype, list] = {}
        cur_bytes: Dict[torch.dtype, int] = {}

        def flush(dt=None):
            for d in ([dt] if dt is not None else list(cur)):
                if cur.get(d):
                    self.buckets.append(_Bucket(cur[d], device))
                cur.pop(d, None)
                cur_bytes.pop(d, None)

        for p in params:
            if id(p) in blocked:
                flush()
                b = _Bucket([p], device)
                b.blocks = blocked[id(p)][1]
                self.buckets.append(b)
                continue
            cur.setdefault(p.dtype, []).append(p)
            cur_bytes[p.dtype] = cur_bytes.get(p.dtype, 0) + p.numel() * p.element_size()
            if cur_bytes[p.dtype] >= bucket_bytes:
                flush(p.dtype)
        flush()
        self.where = {}
        for bi, b in enumerate(self.buckets):
            for p in b.params:
                self.where[id(p)] = bi
        # every averaged parameter, in bucket order, then the NVLS-averaged
        # weights (the ready mask's order)
        self.order = [p for b in self.buckets for p in b.params]
        if self.nvls is not None:
            self.order += self.nvls.params
        pin = device.type == "cuda"
        self._mask_host = torch.zeros(max(1, len(self.order)), dtype=torch.int32, pin_memory=pin)
        self._ready = set()            # ids of parameters marked ready in this step
        self.accumulating = False      # inside no_sync(): gradients accumulate, nothing is reduced
        self.next = 0
        self.armed = False
        self.limited = False
        self.graphed = False
        self.comm_stream = None        # forked stream for reductions captured in a CUDA graph
        self.capture_fork = False
        self.ready_count = 0           # gradients marked ready in this step
        self.launch_marks: List[int] = []   # ready_count at each bucket launch (overlap check)
        apa_params = set()
        for m in mgr.apa_modules.values():
            m._grad_ready_cb = self._apa_ready
            m._dp = self
            apa_params.add(id(m.weight_master))
            if m.bias_master is not None:
                apa_params.add(id(m.bias_master))
        self._hooks = []
        for b in self.buckets:
            for p in b.params:
                if id(p) not in apa_params:
                    self._hooks.append(p.register_post_accumulate_grad_hook(self._param_ready))

    @staticmethod
    def _row_blocks(p, reserved_sms: int, block_rows: int):
        """Row blocks [r0, r1) of a weight gradient [N, K]: whole 256-row tile
        rows, as many as one wave of 256x256 tiles covers on the SMs left
        beside the collective (block_rows overrides)."""
        N, K = p.shape
        rows = block_rows
        if rows <= 0:
            sms = torch.cuda.get_device_properties(p.device).multi_processor_count if p.is_cuda else 148
            clusters = max(1, (sms - max(0, reserved_sms)) // 2)
            rows = 256 * max(1, clusters // max(1, (K + 255) // 256))
        return [(r, min(N, r + rows)) for r in range(0, N, rows)]

    # grads are views into the buckets; re-attach after zero_grad(set_to_none)
    def arm(self):
        for b in self.buckets:
            b.flat.zero_()
            for p in b.params:
                v = b.views[id(p)]
                if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                    p.grad = v
            b.pending = len(b.params)
            b.handles = []
            b.blocks_issued = False
        if self.nvls is not None:
            self.nvls.step_begin()
            for p in self.nvls.params:
                v = self.nvls.views[id(p)]
                if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                    p.grad = v
        self.next = 0
        self.ready_count = 0
        self.launch_marks = []
        self._ready = set()
        self.armed = True

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside accumulate into the buckets without reducing
        them; the next backward outside (the step's last) marks the gradients
        ready and starts the reductions."""
        prev = self.accumulating
        self.accumulating = True
        try:
            yield
        finally:
            self.accumulating = prev

    def _mark(self, p):
        bi = self.where.get(id(p))
        if bi is None or not self.armed or self.accumulating:
            return
        if id(p) in self._ready:
            raise RuntimeError(
                "data parallel: a second backward pass produced gradients after their bucket was reduced; "
                "run every backward pass of a step but the last inside APAManager.no_sync()")
        self._ready.add(id(p))
        b = self.buckets[bi]
        b.pending -= 1
        self.ready_count += 1
        self._launch_ready()

    def _apa_ready(self, mod):
        W = mod.weight_master
        if self.nvls is not None and id(W) in self.nvls.index:
            if self.armed and not self.accumulating:
                if id(W) in self._ready:
                    raise RuntimeError(
                        "data parallel: a second backward pass produced gradients after their reduction started; "
                        "run every backward pass of a step but the last inside APAManager.no_sync()")
                self._ready.add(id(W))
                if id(W) not in self.nvls.fused_now and not self.limited:
                    # the standalone reduction's CTAs need SMs beside the GEMMs
                    self._limit_gemms(True)
                    self.limited = True
                self.nvls.reduce(W)
            if mod.bias_master is not None and mod.bias_master.requires_grad:
                self._mark(mod.bias_master)
            return
        self._mark(mod.weight_master)
        if mod.bias_master is not None and mod.bias_master.requires_grad:
            self._mark(mod.bias_master)

    def _param_ready(self, p):
        bi = self.where.get(id(p))
        if self.armed and bi is not None:
            v = self.buckets[bi].views[id(p)]
            if p.grad is not None and p.grad.data_ptr() != v.data_ptr():
                # produced outside the bucket (the gradient was cleared after
                # pre_step): move it into the bucket, so that every rank
                # reduces it with the bucket's collective
                v.copy_(p.grad)
                p.grad = v
        self._mark(p)

    # parameters that got no gradient this step
    def ready_mask(self) -> torch.Tensor:
        """int32 [len(order)] host tensor: 1 where this rank produced the
        parameter's gradient in the current step (reduce with MAX)."""
        m = self._mask_host
        m.zero_()
        for i, p in enumerate(self.order):
            if id(p) in self._ready:
                m[i] = 1
        return m[:len(self.order)]

    def drop_unused(self, reduced) -> None:
        """After the MAX reduction of every rank's ready_mask(): parameters no
        rank produced a gradient for get grad None (the optimizer skips them,
        as it does on one GPU)."""
        for p, r in zip(self.order, reduced.tolist()):
            if r == 0 and p.grad is not None:
                p.grad = None

    def sync_unused(self) -> None:
        """ready_mask() reduced by its own MAX all-reduce, then drop_unused()
        (for callers that run the averager without the manager, whose
        telemetry reduction carries the mask)."""
        if not self.order:
            return
        dev = self.buckets[0].flat.device
        t = self.ready_mask().to(dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.pg)
        self.drop_unused(t.cpu())

    def _limit_gemms(self, on: bool):
        if self.buckets and self.buckets[0].flat.is_cuda:
            from . import _lib
            n = 0
            if on and self.reserved_sms > 0:
                n = max(1, torch.cuda.get_device_properties(self.buckets[0].flat.device).multi_processor_count
                        - self.reserved_sms)
            _lib.check(_lib.lib().apa_set_gemm_sm_limit(n), "apa_set_gemm_sm_limit")

    def _all_reduce(self, b: _Bucket, t: torch.Tensor):
        if not self.limited:
            self._limit_gemms(True)
            self.limited = True
        op = self.avg_op if self.avg_op is not None else dist.ReduceOp.SUM
        if t.is_cuda and torch.cuda.is_current_stream_capturing():
            # inside a CUDA-graph capture: the reduction runs on a stream forked
            # from the capture stream, so the graph runs it alongside the
            # kernels captured after it; join_capture() joins the fork at the end
            cur = torch.cuda.current_stream(t.device)
            if self.comm_stream is None:
                self.comm_stream = torch.cuda.Stream(device=t.device)
            self.comm_stream.wait_stream(cur)
            with torch.cuda.stream(self.comm_stream):
                dist.all_reduce(t, op=op, group=self.pg)
            self.capture_fork = True
        else:
            b.handles.append(dist.all_reduce(t, op=op, group=self.pg, async_op=True))

    def _launch(self, b: _Bucket):
        self.launch_marks.append(self.ready_count)
        if b.blocks_issued:
            return                    # its row blocks went out during the backward
        self._all_reduce(b, b.flat)

    def grad_view(self, p):
        """p's view into its bucket while a step is armed (for a backward that
        finds p.grad cleared after pre_step), else None."""
        if self.armed and self.nvls is not None and id(p) in self.nvls.index:
            return self.nvls.views[id(p)]
        bi = self.where.get(id(p))
        if not self.armed or bi is None:
            return None
        return self.buckets[bi].views[id(p)]

    def nvls_fused(self, mod, g):
        """The data-parallel arguments for computing mod's weight gradient
        and averaging it over the ranks in one kernel (apa_linear_wgrad_dp),
        or None: only for a gradient of the NVLS buffer, written into its own
        view, while a step is armed and its reduction is due."""
        W = mod.weight_master
        if self.nvls is None or id(W) not in self.nvls.index or not self.armed or self.accumulating:
            return None
        if id(W) in self._ready or g.data_ptr() != self.nvls.views[id(W)].data_ptr():
            return None
        return self.nvls.fused_args(W)

    # row-block reduction of a large APALinear weight (called by its backward)
    def weight_blocks(self, mod, g):
        """The row blocks in which mod's weight gradient is to be computed this
        step, or None: only while armed, with the gradient being the bucket's
        own view and none of its blocks issued yet."""
        W = mod.weight_master
        bi = self.where.get(id(W))
        if not self.armed or bi is None:
            return None
        b = self.buckets[bi]
        if b.blocks is None or b.blocks_issued or g.data_ptr() != b.views[id(W)].data_ptr():
            return None
        return b.blocks

    def weight_block_done(self, mod, r0: int, r1: int):
        """Rows [r0, r1) of mod's weight gradient are written: reduce them."""
        W = mod.weight_master
        b = self.buckets[self.where[id(W)]]
        b.blocks_issued = True
        self._all_reduce(b, b.views[id(W)][r0:r1])

    def join_capture(self, stream):
        """End of a graph capture: the capture stream waits for the forked
        reductions (they must rejoin before the capture ends)."""
        if self.capture_fork:
            stream.wait_stream(self.comm_stream)
            self.capture_fork = False
        if self.nvls is not None:
            self.nvls.join(stream)

    def _launch_ready(self):
        while self.next < len(self.buckets) and self.buckets[self.next].pending <= 0:
            self._launch(self.buckets[self.next])
            self.next += 1

    def graph_captured(self):
        """The step was captured into a CUDA graph: its bucket all-reduces are
        part of the graph and run on every replay, so finish() has nothing
        left to issue or wait for."""
        self.graphed = True
        if self.limited:
            self._limit_gemms(False)
            self.limited = False

    def issue_remaining(self):
        """Issue every bucket not yet issued, in order (asynchronous). Every
        rank must produce every NVLS gradient in every step (the ranks'
        weight-gradient kernels average them region by region with each
        other); a rank that produced none of one raises here, before any other
        collective of the step: models whose layers differ between ranks use
        the NCCL buckets (dp_nvls=False, the default), which reduce a missing
        gradient as zeros."""
        if self.graphed:
            return
        if self.nvls is not None and not self.accumulating:
            missing = [p for p in self.nvls.params if id(p) not in self._ready]
            if missing:
                raise RuntimeError(
                    f"data parallel (dp_nvls=True): {len(missing)} NVLS weight gradient(s) were not produced on this "
                    "rank in this step; every rank must run every APALinear of the NVLS path in every step "
                    "(use dp_nvls=False for models whose layers differ between ranks)")
        while self.next < len(self.buckets):
            self._launch(self.buckets[self.next])
            self.next += 1

    def finish(self):
        """Issue every bucket not yet issued (in order) and make the current
        stream wait for all of them; average when the backend has no AVG.
        Nothing blocks the host: later work on the current stream (the
        optimizer step) runs after the reductions."""
        if self.graphed:
            return
        self.issue_remaining()
        if self.nvls is not None:
            self.nvls.join(torch.cuda.current_stream(self.nvls.buf.device))
        for b in self.buckets:
            for h in b.handles:
                h.wait()
            if self.avg_op is None:
                b.flat.div_(self.world)
            for p in b.params:
                v = b.views[id(p)]
                if p.grad is None:
                    p.grad = v
                elif p.grad.data_ptr() != v.data_ptr():
                    # a gradient assigned directly, not by a backward pass: it
                    # missed its bucket's reduction, and reducing it on its own
                    # here could make the ranks' collectives differ
                    raise RuntimeError(
                        f"data parallel: the gradient of a parameter of shape {tuple(p.shape)} was assigned outside "
                        "the backward pass after pre_step, so it was not averaged")
        if self.limited:
            self._limit_gemms(False)
            self.limited = False
        self.armed = False
