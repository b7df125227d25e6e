"""Data-parallel host logic on CPU with two gloo ranks (no GPU):

* GradientAverager: gradients written into the flat buckets by autograd are
  averaged across ranks, buckets are issued in a fixed order as they fill, and
  zero_grad(set_to_none=True) between steps is handled by re-arming.
* The ladder's telemetry reduction: amax / ratio encoded as int32 bit
  patterns reduce under MAX to the float maximum, with NaN dominating, so every
  rank evaluates the same global values (the reference evaluates local values
  only, manager.py:221-256).
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _FakeManager:
    """The two things GradientAverager reads from APAManager."""

    def __init__(self, model):
        self.model = model
        self.apa_modules = {}

    def get_trainable_parameters(self):
        return [p for p in self.model.parameters() if p.requires_grad]


def _averager_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from apa.dp import GradientAverager
        def build():
            torch.manual_seed(0)                   # identical weights on both ranks
            return nn.Sequential(nn.Linear(6, 5), nn.ReLU(), nn.Linear(5, 3), nn.LayerNorm(3))

        model, plain = build(), build()            # plain: same model without the averager
        avg = GradientAverager(_FakeManager(model), None, bucket_bytes=64)   # several small buckets
        results = []
        for step in range(3):
            g = torch.Generator().manual_seed(100 * step + rank)          # different data per rank
            x = torch.randn(4, 6, generator=g)
            plain(x).pow(2).sum().backward()
            local = [p.grad.clone() for p in plain.parameters()]
            for p in plain.parameters():
                p.grad = None
            avg.arm()
            model(x).pow(2).sum().backward()
            issued_before_finish = avg.next
            avg.finish()
            results.append(([p.grad.tolist() for p in model.parameters()], [t.tolist() for t in local],
                            issued_before_finish, len(avg.buckets)))
            for p in model.parameters():
                p.grad = None                      # zero_grad(set_to_none=True)
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_gradient_averager_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_averager_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for step in range(3):
        avg0, local0, issued0, nb = out[0][step]
        avg1, local1, issued1, _ = out[1][step]
        assert nb > 1
        assert issued0 == issued1 == nb            # every bucket issued by the hooks, in order
        for a0, a1, l0, l1 in zip(avg0, avg1, local0, local1):
            a0, a1, l0, l1 = (torch.tensor(v) for v in (a0, a1, l0, l1))
            want = (l0 + l1) / 2
            assert torch.allclose(a0, want, atol=1e-6) and torch.equal(a0, a1)


class _ApaFirstManager(_FakeManager):
    """Lists parameters the way APAManager.get_trainable_parameters does:
    the layers it manages first, every other parameter after."""

    def get_trainable_parameters(self):
        ps = list(self.model.parameters())
        return ps[2:] + ps[:2]


def _order_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from apa.dp import GradientAverager
        torch.manual_seed(0)
        # an embedding registered first: its gradient is produced last by backward
        model = nn.Sequential(nn.Embedding(50, 16), nn.Linear(16, 16), nn.ReLU(), nn.Linear(16, 8))
        avg = GradientAverager(_ApaFirstManager(model), None, bucket_bytes=256)
        avg.arm()
        idx = torch.randint(0, 50, (12,), generator=torch.Generator().manual_seed(rank))
        model(idx).pow(2).sum().backward()
        marks, total = list(avg.launch_marks), avg.ready_count
        sizes = [len(b.params) for b in avg.buckets]
        avg.finish()
        q.put((rank, marks, total, sizes))
    finally:
        dist.destroy_process_group()


def test_buckets_follow_backward_order_two_ranks():
    """Buckets are issued strictly in order; the first one must go out before
    the last gradient exists (buckets built from the manager's listing would
    put the embedding first and hold every reduction to the end of backward)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_order_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        marks, total, sizes = out[r]
        assert len(sizes) > 2 and len(marks) == len(sizes)
        # each bucket goes out as soon as its own gradients exist (weight and
        # bias of one layer may arrive in either order)
        cum = 0
        for m, n in zip(marks, sizes):
            cum += n
            assert m <= cum + 1, (marks, sizes)
        assert marks[0] < total


class _FakeApaLinear(nn.Module):
    """The attributes GradientAverager and the row-block path use."""

    def __init__(self, n, k):
        super().__init__()
        self.weight_master = nn.Parameter(torch.randn(n, k))
        self.bias_master = nn.Parameter(torch.randn(n))
        self._grad_ready_cb = None
        self._dp = None


class _ApaManager(_FakeManager):
    def __init__(self, model, mods):
        super().__init__(model)
        self.apa_modules = mods


def _blocks_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from apa.dp import GradientAverager
        torch.manual_seed(0)
        big, small = _FakeApaLinear(10, 6), _FakeApaLinear(4, 6)
        model = nn.ModuleDict({"small": small, "big": big})
        avg = GradientAverager(_ApaManager(model, {"small": small, "big": big}), None, bucket_bytes=1 << 20,
                               block_bytes=200, block_rows=3)
        out = {"blocked": [big._dp is avg and avg.buckets[avg.where[id(big.weight_master)]].blocks is not None,
                           avg.buckets[avg.where[id(small.weight_master)]].blocks is None]}
        W = big.weight_master
        for step in range(2):
            avg.arm()
            local = {r: torch.randn(10, 6, generator=torch.Generator().manual_seed(10 * step + r)) for r in range(world)}
            local_s = {r: torch.randn(4, 6, generator=torch.Generator().manual_seed(99 + 10 * step + r))
                       for r in range(world)}
            # the big layer's backward: its gradient in row blocks
            blocks = avg.weight_blocks(big, W.grad)
            out["blocks"] = blocks
            for r0, r1 in blocks:
                W.grad[r0:r1] = local[rank][r0:r1]
                avg.weight_block_done(big, r0, r1)
            out["again"] = avg.weight_blocks(big, W.grad)        # no second pass in one step
            big.bias_master.grad.fill_(float(rank))
            big._grad_ready_cb(big)
            small.weight_master.grad.copy_(local_s[rank])
            small.bias_master.grad.fill_(2.0 * rank)
            small._grad_ready_cb(small)
            nh = [len(b.handles) for b in avg.buckets]
            avg.finish()
            want = sum(local.values()) / world
            want_s = sum(local_s.values()) / world
            out[f"step{step}"] = (torch.equal(W.grad, want), torch.allclose(small.weight_master.grad, want_s),
                                  big.bias_master.grad[0].item(), small.bias_master.grad[0].item(), nh)
        out["unarmed"] = avg.weight_blocks(big, W.grad)
        # the bucket view a backward writes into when the gradient was cleared
        out["view_unarmed"] = avg.grad_view(W) is None
        avg.arm()
        v = avg.grad_view(W)
        out["view_armed"] = v is not None and v.data_ptr() == W.grad.data_ptr() and v.shape == W.shape
        out["view_foreign"] = avg.grad_view(torch.nn.Parameter(torch.zeros(3))) is None
        avg.finish()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_block_reduction_two_ranks():
    """A large APALinear weight sits alone in its bucket and is reduced block
    by block as its backward writes the rows; the bucket is not reduced again,
    and every gradient ends up averaged exactly once."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_blocks_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        o = out[r]
        assert o["blocked"] == [True, True]
        assert o["blocks"] == [(0, 3), (3, 6), (6, 9), (9, 10)]
        assert o["again"] is None and o["unarmed"] is None
        assert o["view_unarmed"] and o["view_armed"] and o["view_foreign"]
        for step in (0, 1):
            ok_w, ok_s, bb, sb, nh = o[f"step{step}"]
            assert ok_w and ok_s
            assert bb == 0.5 and sb == 1.0
            # buckets in backward order: [big bias], [big weight: 4 blocks], [small bias + weight]
            assert nh == [1, 4, 1]


def _telemetry_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vals = {0: [0.5, 3.0, 0.0, float("inf"), 1.0], 1: [2.0, float("nan"), 0.25, 7.0, 0.0]}[rank]
        t = torch.tensor(vals, dtype=torch.float32).view(torch.int32).clone()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, t.view(torch.float32).tolist()))
    finally:
        dist.destroy_process_group()


def test_telemetry_bit_pattern_max_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_telemetry_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        v = out[r]
        assert v[0] == 2.0 and math.isnan(v[1]) and v[2] == 0.25 and math.isinf(v[3]) and v[4] == 1.0


def _run_two(worker):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


class _MixedModel(nn.Module):
    """fp32 linear layers, a bf16 LayerNorm and an fp16 scale vector, and a
    branch (`extra`) used only when asked."""

    def __init__(self):
        super().__init__()
        self.a = nn.Linear(6, 8)
        self.norm = nn.LayerNorm(8).to(torch.bfloat16)
        self.scale = nn.Parameter(torch.ones(8, dtype=torch.float16))
        self.b = nn.Linear(8, 3)
        self.extra = nn.Linear(8, 3)

    def forward(self, x, use_extra=False):
        h = self.norm(self.a(x).to(torch.bfloat16)).float() * self.scale.float()
        y = self.b(h)
        return y + self.extra(h) if use_extra else y


def _mixed_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from apa.dp import GradientAverager
        torch.manual_seed(0)
        model = _MixedModel()
        avg = GradientAverager(_FakeManager(model), None, bucket_bytes=64)
        out = {"dtypes": sorted({str(b.dtype) for b in avg.buckets}),
               "covered": all(id(p) in avg.where for p in model.parameters())}
        # step 1: `extra` unused on both ranks; the caller clears the gradients
        # after arming (zero_grad(set_to_none=True) after pre_step)
        x = torch.randn(4, 6, generator=torch.Generator().manual_seed(rank))
        avg.arm()
        for p in model.parameters():
            p.grad = None
        model(x).pow(2).sum().backward()
        avg.finish()
        avg.sync_unused()
        out["step1"] = {n: (None if p.grad is None else p.grad.float().tolist()) for n, p in model.named_parameters()}
        out["in_bucket"] = all(p.grad is None or p.grad.data_ptr() == avg.buckets[avg.where[id(p)]].views[id(p)]
                               .data_ptr() for p in model.parameters())
        # step 2: `extra` used on rank 1 only
        avg.arm()
        model(x, use_extra=(rank == 1)).pow(2).sum().backward()
        avg.finish()
        avg.sync_unused()
        out["step2_extra"] = None if model.extra.weight.grad is None else model.extra.weight.grad.tolist()
        # the local gradients of each step, for the expected averages
        ref = _MixedModel()
        ref.load_state_dict(model.state_dict())
        ref(x).pow(2).sum().backward()
        out["local1"] = {n: p.grad.float().tolist() for n, p in ref.named_parameters() if p.grad is not None}
        ref.zero_grad(set_to_none=True)
        ref(x, use_extra=(rank == 1)).pow(2).sum().backward()
        out["local2_extra"] = None if ref.extra.weight.grad is None else ref.extra.weight.grad.tolist()
        # gradient accumulation: a second backward outside no_sync raises;
        # inside it the micro-batches accumulate and the last one reduces
        avg.arm()
        model(x).sum().backward()
        try:
            model(x).sum().backward()
            out["double"] = "no error"
        except RuntimeError as e:
            out["double"] = "raised" if "no_sync" in str(e) else str(e)
        avg.finish()
        avg.arm()
        with avg.no_sync():
            model(x).sum().backward()
        model(2 * x).sum().backward()
        avg.finish()
        out["accum_a"] = model.a.weight.grad.tolist()
        ref.zero_grad(set_to_none=True)
        ref(x).sum().backward()
        ref(2 * x).sum().backward()
        out["local_accum_a"] = ref.a.weight.grad.tolist()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_mixed_dtypes_unused_and_accumulation_two_ranks():
    """Every trainable parameter is averaged, whatever its dtype (bf16 and fp16
    parameters get buckets of their own); a gradient produced outside its
    bucket (cleared after arming) is still reduced with it; a parameter no
    rank used ends the step with grad None, one used by a single rank gets the
    average; a second backward outside no_sync() raises, and micro-batches
    under no_sync() accumulate before the one reduction."""
    out = _run_two(_mixed_worker)
    for r in (0, 1):
        o = out[r]
        assert o["dtypes"] == ["torch.bfloat16", "torch.float16", "torch.float32"]
        assert o["covered"] and o["in_bucket"]
        assert o["step1"]["extra.weight"] is None and o["step1"]["extra.bias"] is None
        assert o["double"] == "raised"
    for name in ("a.weight", "a.bias", "norm.weight", "norm.bias", "scale", "b.weight", "b.bias"):
        g0, g1 = torch.tensor(out[0]["step1"][name]), torch.tensor(out[1]["step1"][name])
        assert torch.equal(g0, g1), name                       # replicas agree
        want = (torch.tensor(out[0]["local1"][name]) + torch.tensor(out[1]["local1"][name])) / 2
        tol = 1e-5 if name.startswith(("a.", "b.")) else 2e-2  # bf16 / fp16 buckets
        assert torch.allclose(g0, want, rtol=tol, atol=tol), name
    e0, e1 = torch.tensor(out[0]["step2_extra"]), torch.tensor(out[1]["step2_extra"])
    assert torch.equal(e0, e1) and out[0]["local2_extra"] is None
    assert torch.allclose(e0, torch.tensor(out[1]["local2_extra"]) / 2, atol=1e-6)
    a0 = torch.tensor(out[0]["accum_a"])
    want = (torch.tensor(out[0]["local_accum_a"]) + torch.tensor(out[1]["local_accum_a"])) / 2
    assert torch.equal(a0, torch.tensor(out[1]["accum_a"])) and torch.allclose(a0, want, atol=1e-5)


class _FakeNvls:
    """Stands in for the NVLS gradient buffer (which needs CUDA symmetric
    memory): the host-side bookkeeping GradientAverager keeps for it."""

    def __init__(self, params):
        self.params = list(params)
        self.index = {id(p): i for i, p in enumerate(self.params)}
        self.views = {id(p): torch.zeros_like(p) for p in self.params}
        self.fused_now = set()
        self.reduced = []

    def step_begin(self):
        self.fused_now.clear()

    def reduce(self, p):
        self.reduced.append(id(p))

    def join(self, stream):
        pass


def _nvls_missing_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from apa.dp import GradientAverager
        torch.manual_seed(0)
        model = nn.Linear(8, 8, bias=False)
        avg = GradientAverager(_FakeManager(model), None)
        avg.nvls = _FakeNvls([model.weight])
        avg.buckets, avg.next = [], 0       # only the NVLS gradient: no collective in this test
        out = {}
        avg.arm()
        if rank == 0:
            avg._ready.add(id(model.weight))   # this rank's backward produced it
        try:
            avg.issue_remaining()
            out["raised"] = None
        except RuntimeError as e:
            out["raised"] = str(e)
        # inside no_sync the gradients are not reduced yet: nothing is checked
        avg.arm()
        with avg.no_sync():
            avg.issue_remaining()
        out["no_sync_ok"] = True
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_nvls_gradient_missing_on_a_rank_raises():
    """With the NVLS path every rank must produce every NVLS gradient in every
    step (the ranks' kernels average them region by region); a rank that did
    not raises at the end of its backward, before issuing any collective."""
    out = _run_two(_nvls_missing_worker)
    assert out[0]["raised"] is None
    assert out[1]["raised"] is not None and "dp_nvls=False" in out[1]["raised"]
    assert out[0]["no_sync_ok"] and out[1]["no_sync_ok"]
