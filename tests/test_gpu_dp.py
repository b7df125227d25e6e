"""Data parallel on 2+ GPUs (skipped with fewer): ranks that see different
data take identical decisions.

Each rank trains the same small model on its own batches; at one step only
rank 1's batch carries an overflow spike. The reference evaluates local
telemetry only (manager.py:221-256), so its ranks would disagree; here the
telemetry is MAX-reduced before the ladder and the gradients are averaged, so
every rank must skip that step, escalate the same layers, and keep
bit-identical weights. With row blocks on, the first layer's weight gradient
is computed and all-reduced in four row blocks; the replicas must then equal
those of the whole-bucket reduction bit for bit. NVLS is disabled so a rank
that fails an assertion cannot leave a multicast binding behind."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 8
SPIKE_STEP = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, graphed, blocks):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    from datetime import timedelta
    import torch.distributed as dist
    import torch.nn as nn
    import torch.nn.functional as F
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "adaptive-precision-ascension_b200"))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from apa import APAConfig, APALinear, APAManager
        class LayerNorm32(nn.LayerNorm):   # takes the fp16 output of an escalated layer
            def forward(self, x):
                return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps)

        cfg = APAConfig(device=str(dev), check_interval=2)
        torch.manual_seed(0)
        model = nn.Sequential(APALinear(256, 256, config=cfg), nn.ReLU(), LayerNorm32(256),
                              APALinear(256, 16, config=cfg)).to(dev)
        mgr = APAManager(model, cfg, dp_block_bytes=1 if blocks else 0, dp_block_rows=64)
        opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=1e-3)
        g = torch.Generator().manual_seed(100 + rank)
        keeps, levels = [], []
        xs = torch.empty(128, 256, device=dev)
        ys = torch.empty(128, dtype=torch.long, device=dev)
        gstep = None
        if graphed:
            from apa.graphs import GraphedTrainStep
            gstep = GraphedTrainStep(mgr, lambda a, b: F.cross_entropy(model(a), b), (xs, ys), warmup=2,
                                     static_inputs=True)
        for step in range(STEPS):
            x = torch.randn(128, 256, generator=g)
            y = torch.randint(0, 16, (128,), generator=g)
            if step == SPIKE_STEP and rank == 1:
                idx = torch.randperm(x.numel(), generator=g)[:64]
                x.view(-1)[idx] *= 1e3
            xs.copy_(x)
            ys.copy_(y)
            if gstep is not None:
                _, keep = gstep(xs, ys)
            else:
                mgr.pre_step()
                opt.zero_grad(set_to_none=True)
                F.cross_entropy(model(xs), ys).backward()
                keep = mgr.post_backward_sync_and_eval()
            if keep:
                opt.step()
            keeps.append(bool(keep))
            levels.append([m.level for m in mgr.apa_modules.values()])
        torch.cuda.synchronize()
        gstep = None   # a graph holding NCCL work is released before the group
        used = [len(b.blocks) for b in mgr._dp.buckets if b.blocks is not None and b.blocks_issued]
        weights = [p.detach().double().cpu() for p in mgr.get_trainable_parameters()]
        q.put((rank, keeps, levels, [w.sum().item() for w in weights], [w.abs().sum().item() for w in weights],
               used))
    except Exception as e:   # report, then leave the group normally
        q.put((rank, "error", repr(e), None, None, None))
    finally:
        dist.destroy_process_group()


def _run(graphed, blocks, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, graphed, blocks)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict((r[0], r[1:]) for r in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert out[r][0] != "error", out[r]
    keeps0, levels0, sums0, abs0, used0 = out[0]
    for r in range(1, world):
        keeps, levels, sums, abss, used = out[r]
        assert keeps == keeps0
        assert levels == levels0
        assert sums == sums0 and abss == abs0     # bit-identical replicas
        assert used == used0
    assert keeps0[SPIKE_STEP] is False            # only rank 1 saw the spike; every rank skips
    assert all(keeps0[s] for s in range(STEPS) if s != SPIKE_STEP)
    assert levels0[SPIKE_STEP][0] == 1            # the first layer escalated on every rank
    return out[0]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("graphed", [False, True])
def test_ranks_take_identical_decisions(graphed):
    """graphed: the step replayed from a CUDA graph (reductions captured on a
    forked stream, ladder gated on the step's compute)."""
    assert _run(graphed, blocks=False)[4] == []


@pytest.mark.parametrize("world", [4, 8])
def test_ranks_take_identical_decisions_wider(world):
    """The same check with 4 and 8 ranks (only rank 1 sees the spike), where
    the box has that many GPUs."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    assert _run(False, blocks=False, world=world)[4] == []


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("graphed", [False, True])
def test_row_block_reduction_matches_whole(graphed):
    """The first layer's 256x256 weight gradient in four 64-row blocks, each
    all-reduced as soon as it is written: same decisions and bit-identical
    weights as the whole-bucket reduction."""
    whole = _run(graphed, blocks=False)
    blocked = _run(graphed, blocks=True)
    assert blocked[4] == [4]
    assert blocked[:4] == whole[:4]
