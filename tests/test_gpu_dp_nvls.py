"""Data-parallel weight gradients averaged through NVLink SHARP (the region
protocol: apa_linear_wgrad_dp, whose epilogue publishes every 32 x 64 region
of the gradient as it is stored and averages the regions its rank owns with
multimem.ld_reduce / multimem.st, and the standalone apa_dp_region_signal /
apa_dp_region_reduce for gradients written otherwise) against the NCCL bucket
path, on 2 GPUs (skipped with fewer, or where the GPUs have no NVLink
multicast).

Each rank trains the same model on its own batches for a few AdamW steps,
once with the NVLS path and once with NCCL buckets only:

* fused: a 2048 x 2048 APALinear (large enough for the NVLS path; its weight
  gradient is one GEMM, so the GEMM's epilogue runs the reduction), then a
  small one;
* split: a 1024 x 1024 APALinear over 8192 tokens, whose weight gradient is
  split along the tokens (two kernels), so the standalone kernels reduce it
  inside apa_linear_wgrad_dp;

At the FP8 rung the per-rank gradients are E4M3 values, whose sums over a few
ranks are exact in fp32, so both paths average to the same bits and the
weights after training are identical; at FP16 and TF32 the two reductions add
in different orders, so the weights agree to fp32 rounding. In every case the
ranks' replicas are bit-identical to each other. Eager and graph-replayed
steps."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(case, cfg, dev, rank):
    import torch.nn as nn
    from apa import APALinear

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            d = 1024 if case == "split" else 2048
            self.a = APALinear(d, d, config=cfg)
            self.head = APALinear(d, 16, config=cfg)

        def forward(self, x):
            return self.head(torch.relu(self.a(x)))

    return Net().to(dev)


def _worker(rank, world, port, q, case, level, graphed):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    from datetime import timedelta
    import torch.distributed as dist
    import torch.nn.functional as F
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "adaptive-precision-ascension_b200"))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from apa import APAConfig, APALinear, APAManager
        out = {}
        tokens = 8192 if case == "split" else 256
        d = 1024 if case == "split" else 2048
        for nvls in (True, False):
            cfg = APAConfig(device=str(dev), check_interval=4)
            torch.manual_seed(0)
            model = _model(case, cfg, dev, rank)
            for m in model.modules():
                if isinstance(m, APALinear):
                    m.level = level
            mgr = APAManager(model, cfg, dp_nvls=nvls)
            opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=1e-3)
            g = torch.Generator().manual_seed(100 + rank)
            xs = torch.empty(tokens, d, device=dev)
            ys = torch.empty(tokens, dtype=torch.long, device=dev)
            gstep = None
            if graphed:
                from apa.graphs import GraphedTrainStep
                gstep = GraphedTrainStep(mgr, lambda a, b: F.cross_entropy(model(a).float(), b), (xs, ys),
                                         warmup=2, static_inputs=True)
            keeps = []
            for step in range(STEPS):
                xs.copy_(torch.randn(tokens, d, generator=g))
                ys.copy_(torch.randint(0, 16, (tokens,), generator=g))
                if gstep is not None:
                    _, keep = gstep(xs, ys)
                else:
                    mgr.pre_step()
                    opt.zero_grad(set_to_none=True)
                    F.cross_entropy(model(xs).float(), ys).backward()
                    keep = mgr.post_backward_sync_and_eval()
                if keep:
                    opt.step()
                keeps.append(bool(keep))
            torch.cuda.synchronize()
            gstep = None
            nv = mgr._dp.nvls
            out[nvls] = dict(used=nv is not None, fused=nv.fused_calls if nv else 0,
                             standalone=nv.standalone_calls if nv else 0, keeps=keeps,
                             w=[p.detach().double().cpu() for p in mgr.get_trainable_parameters()])
            del mgr, opt, model
            torch.cuda.synchronize()
        from apa import _lib
        status = _lib.device_status()
        q.put((rank, {k: dict(used=v["used"], fused=v["fused"], standalone=v["standalone"], keeps=v["keeps"],
                              sums=[float(w.sum()) for w in v["w"]], abs=[float(w.abs().sum()) for w in v["w"]],
                              maxdiff=[float((a - b).abs().max()) for a, b in zip(v["w"], out[False]["w"])])
                      for k, v in out.items()}, status))
    except Exception as e:   # report, then leave the group normally
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _run(case, level, graphed, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, case, level, graphed)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][0] != "error", res[r]
    return res


CASES = [("fused", 0, False), ("fused", 0, True), ("fused", 1, False), ("fused", 1, True), ("fused", 2, False),
         ("fused", 2, True), ("split", 0, False), ("split", 0, True), ("split", 2, False)]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case,level,graphed", CASES)
def test_nvls_average_matches_nccl(case, level, graphed):
    res = _run(case, level, graphed)
    out0, status0 = res[0]
    if not out0[True]["used"]:
        pytest.skip("no NVLink multicast on these GPUs: the NCCL buckets carry every gradient")
    for r in res:
        out, status = res[r]
        assert status == 0
        assert out[True]["used"] and not out[False]["used"]
        assert out[True]["keeps"] == out[False]["keeps"] == [True] * STEPS
        # replicas identical across ranks, on each path
        assert out[True]["sums"] == out0[True]["sums"] and out[True]["abs"] == out0[True]["abs"]
        assert out[False]["sums"] == out0[False]["sums"]
        if level == 0:
            assert max(out[True]["maxdiff"]) == 0.0      # exact sums of E4M3 gradients
        else:
            assert max(out[True]["maxdiff"]) < 1e-5
        if not graphed:
            assert out[True]["fused"] > 0     # the GEMM's epilogue reduced the large gradient
