"""Benchmark: APALinear forward+backward TFLOP/s per ladder rung.

Workload (default): one APALinear at M=8192 tokens, K=4096, N=4096 with fp32
master weights (Kaiming-uniform, seed 0), bf16 activations ~ N(0,1) (seed 0)
and upstream gradients ~ N(0,1) (seed 1; fp32 at the FP8/TF32 rungs, fp16 at
the FP16 rung, the output dtype). A step is the reference's full training
step for that layer through the public API: APAManager.pre_step (working
copy), forward, backward, post_backward_sync_and_eval (ladder + the one host
read); 6*M*N*K FLOPs per step. The headline `value` is the FP8 rung.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (launched by torchrun, one rank per GPU, NCCL) every rank runs the
same layer on its own 8192-token shard (weak scaling) and the step includes the
data-parallel gradient all-reduce and the telemetry all-reduce; `value` is the
whole-job FLOP rate with time taken as the max over ranks.

`--impl reference` times the reference's own implementation of the path, its
fp8_simulation_mode CPU path, on this host's cores, FP8 rung, on a bounded
number of full steps, plus the cfg0 quick-start MLP's 200 steps: the reference
package when it is installed under baseline/_ref, else the torch-CPU port of
that path (oracle/ref_port.py, bit-exact against the reference's own outputs);
`cpu_baseline.kind` says which ran.

Besides the headline, the JSON line carries: `rungs` (all three rungs),
`roofline` (the FP8 forward GEMM timed alone, with the fused-telemetry cost),
`optimizer` (the fused AdamW + working-copy kernel on the 4096x4096 master
against torch's fused AdamW plus the cast), `e2e` (host-resident inputs copied
every step), `gpt` (char nanoGPT and GPT-2-medium tokens/s) and `vit` (the ViT
classifier's images/s), all at the same N; `cpu_baseline` and `cfg0` (the
quick-start MLP's steps/s through this library) at N=1.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "adaptive-precision-ascension_b200")

M, K, N = 8192, 4096, 4096
FLOPS_STEP = 6.0 * M * N * K
METRIC = "APALinear fwd+bwd TFLOP/s (FP8 rung)"
CONFIG = {"workload": "APALinear 8192x4096x4096 fwd+bwd, full APA step (pre_step, fwd, bwd, ladder)",
          "M": M, "K": K, "N": N, "x": "bf16 N(0,1) seed 0", "dy": "N(0,1) seed 1, output dtype",
          "l2": "inputs larger than L2: ~0.8 GB touched per step vs 126 MB L2"}


def peaks():
    p = {"source": "fallback", "hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        p = {"source": "measured", "hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"]}
    # dense FP8 runs at twice the dense bf16 rate on B200; TF32 at half
    p["fp8_tflops"] = 2.0 * p["bf16_tflops"]
    p["fp16_tflops"] = p["bf16_tflops"]
    p["tf32_tflops"] = 0.5 * p["bf16_tflops"]
    return p


def library_peaks(torch, dev):
    """Dense GEMM throughput of the vendor libraries on this GPU, a second
    reference for the rung rooflines: cuBLASLt FP8 (torch._scaled_mm, E4M3 x
    E4M3, unit scales, bf16 out), cuBLAS fp16 and TF32 (fp32 inputs with TF32
    math) at 8192^3, best of a few back-to-back launches (burst, like the bf16
    figure of MEASURED_PEAKS.json)."""
    n = 8192
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    a32 = torch.randn(n, n, device=dev, generator=g)
    b32 = torch.randn(n, n, device=dev, generator=g)

    def best(fn, reps=10):
        for _ in range(3):
            fn()
        t = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            t.append(e0.elapsed_time(e1))
        return 2.0 * n ** 3 / (min(t) * 1e-3) / 1e12

    try:
        a8, b8 = a32.to(torch.float8_e4m3fn), b32.to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        out["fp8_tflops"] = round(best(lambda: torch._scaled_mm(a8, b8, scale_a=one, scale_b=one,
                                                                out_dtype=torch.bfloat16)), 1)
    except Exception as e:   # the library path is only a reference denominator
        out["fp8_error"] = repr(e)[:120]
    a16, b16 = a32.half(), b32.half()
    out["fp16_tflops"] = round(best(lambda: a16 @ b16), 1)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    out["tf32_tflops"] = round(best(lambda: a32 @ b32), 1)
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a32, b32
    torch.cuda.empty_cache()
    return out


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
def grad_allreduce_desc(args):
    if args.dp_nvls:
        return ("APALinear weights of 1 Mi elements or more averaged through NVLink SHARP (multimem) where the GPUs "
                "have it, the rest in NCCL buckets")
    if args.dp_block_bytes > 0:
        return f"NCCL, row blocks for weights >= {args.dp_block_bytes} B"
    return "NCCL, whole buckets"


def gpt_optimizer(args, name: str) -> str:
    """The GPT workload's optimizer: "auto" takes the library's fused AdamW
    (master update + next step's working copies in one pass) for GPT-2-medium,
    where it measured level with or faster than torch's fused AdamW followed by
    the casts, and torch's fused AdamW for the char model, whose many small
    weights make one launch per weight cost more than the pass saves."""
    if args.gpt_optimizer != "auto":
        return args.gpt_optimizer
    return "apa" if name == "gpt2m" else "torch"


def run_ours(args):
    sys.path.insert(0, PKG)
    import torch
    import torch.distributed as dist
    import torch.nn as nn
    from apa import APAConfig, APALinear, APAManager, _lib

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _lib.check(_lib.lib().apa_set_pdl(0 if args.no_pdl else 1), "apa_set_pdl")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    g = torch.Generator(device=dev).manual_seed(0 + 1000 * rank)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    g1 = torch.Generator(device=dev).manual_seed(1 + 1000 * rank)
    dy32 = torch.randn(M, N, device=dev, generator=g1)
    dy16 = dy32.half()

    def make(level):
        cfg = APAConfig(device=str(dev), check_interval=1)
        torch.manual_seed(0)
        lin = APALinear(K, N, config=cfg)
        lin.level = level
        mgr = APAManager(nn.Sequential(lin), cfg, bucket_bytes=args.dp_bucket_bytes,
                         dp_block_bytes=args.dp_block_bytes, dp_nvls=bool(args.dp_nvls))
        return lin, mgr

    results = {}
    gemm_roof = None
    optim = None
    launches = 0
    clocks = None
    pk = peaks()
    libpk = library_peaks(torch, dev) if rank == 0 else {}
    gstep = None
    from apa.graphs import GraphedTrainStep
    for level, name in ((0, "fp8"), (1, "fp16"), (2, "tf32")):
        lin, mgr = make(level)
        dy = dy16 if level == 1 else dy32
        xr = x.detach().requires_grad_(True)

        if args.eager:
            def step():
                mgr.pre_step()
                y = lin(xr)
                y.backward(dy)
                xr.grad = None
                return mgr.post_backward_sync_and_eval()
        else:
            # pre_step + forward + backward replayed from a CUDA graph (the
            # inputs stay in place), ladder decision eager: every step runs
            # the same kernels as the eager path, minus the host launch work
            gstep = GraphedTrainStep(mgr, lambda xx, gg: (lin(xx), gg), (xr, dy), warmup=2, static_inputs=True)

            def step():
                return gstep(xr, dy)[1]

        # the clock sampler starts before the warm-up (its process start-up
        # stays out of the timed region) and runs through the timed steps
        sampler = ClockSampler(local) if (level == 0 and rank == 0) else None
        if sampler:
            sampler.__enter__()
        for _ in range(args.warmup):
            step()
        barrier()
        c0 = _lib.calls
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            step()
        e1.record(s)
        barrier()
        if sampler:
            sampler.__exit__()
            clocks = sampler.summary()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        if level == 0:
            # library launches in the timed steps: the ones issued from the host
            # plus those inside each replayed graph
            launches = (_lib.calls - c0) + (0 if args.eager else args.steps * gstep.captured_launches)
        results[name] = {"ms_per_step": ms, "tflops": world * FLOPS_STEP / ms / 1e9,
                         "frac_of_peak": FLOPS_STEP / ms / 1e9 / pk[f"{name}_tflops"]}
        if f"{name}_tflops" in libpk:
            results[name]["frac_of_library_gemm"] = FLOPS_STEP / ms / 1e9 / libpk[f"{name}_tflops"]
        if level == 0:
            gemm_roof = time_gemm(torch, _lib, lin, xr, dev, pk, libpk)
            optim = time_optimizer(torch, _lib, dev, pk)
        # graphs holding NCCL work must be released before the process group
        gstep = step = None
        del lin, mgr
        torch.cuda.empty_cache()

    # end to end: host-resident inputs, copied in every step, result read back
    e2e = run_e2e(torch, make, x, dy32, dev, args, world, barrier, max_over_ranks)
    del x, dy32, dy16
    torch.cuda.empty_cache()
    gpt = {}
    vit = None
    if args.vit:
        vit = run_vit(torch, world, rank, dev, args.gpt_steps, max(4, args.warmup), barrier, max_over_ranks,
                      graphed=not args.gpt_eager, dp_bucket_bytes=args.dp_bucket_bytes, dp_nvls=bool(args.dp_nvls))
    for name in args.gpt:
        gpt[name] = run_gpt(torch, dist, name, world, rank, dev, args.gpt_steps, max(4, args.warmup), barrier,
                            max_over_ranks, graphed=not args.gpt_eager, optimizer=gpt_optimizer(args, name),
                            dp_block_bytes=args.dp_block_bytes, dp_bucket_bytes=args.dp_bucket_bytes,
                            dp_nvls=bool(args.dp_nvls))
    out = None
    if rank == 0:
        fp8 = results["fp8"]
        out = {
            "metric": METRIC, "value": round(fp8["tflops"], 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(fp8["ms_per_step"], 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic", "config": dict(CONFIG, parallelism=f"dp{world}",
                                                launch=("eager" if args.eager else
                                                        "cuda-graph replay of pre_step+fwd+bwd, ladder eager")
                                                + ("" if args.no_pdl else
                                                   ", programmatic dependent launch between the library's kernels"),
                                                grad_allreduce=grad_allreduce_desc(args)),
            "rungs": {k: {"tflops": round(v["tflops"], 2), "ms_per_step": round(v["ms_per_step"], 4),
                          "frac_of_peak": round(v["frac_of_peak"], 4),
                          "frac_of_library_gemm": round(v.get("frac_of_library_gemm", 0.0), 4)}
                      for k, v in results.items()},
            "library_gemm_peaks": libpk,
            "roofline": gemm_roof,
            "optimizer": optim,
            "e2e": e2e,
            "gpt": gpt,
            "vit": vit,
            "gpu_launches": launches,
            "clocks": clocks,
            "peaks": pk,
        }
        if world == 1:
            out["cfg0"] = cfg0_gpu(torch, dev)
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(args, sample_steps=1)
    if world > 1:
        dist.destroy_process_group()
    return out



# ---------------------------------------------------------------------------
# GPT training workloads (harness: the model around the APALinear layers)
# ---------------------------------------------------------------------------
GPT_CONFIGS = {
    # char-level nanoGPT: 6 layers, 6 heads, d 384, context 256, vocab 65,
    # per-GPU batch 64, uniform tokens, AdamW 1e-3, default config
    "gpt-char": dict(n_layer=6, n_head=6, d=384, T=256, vocab=65, vocab_pad=65, batch=64, lr=1e-3,
                     zipf=None, preset="default", preset_levels=False),
    # GPT-2-medium shape: 24 layers, 16 heads, d 1024, context 1024, vocab
    # 50257, per-GPU batch 8, Zipf(1.1) tokens, aggressive() config, QKV of
    # layers 0-3 at FP16 and the LM head at TF32 from the start. The LM head
    # has 50304 outputs (16-byte aligned rows); the 47 extra classes carry a
    # -30000 bias in fp32 (the head starts at TF32 and the ladder only moves
    # up), so their softmax probability and gradients are exactly zero and the
    # model computes the 50257-class function without slicing the logits.
    "gpt2m": dict(n_layer=24, n_head=16, d=1024, T=1024, vocab=50257, vocab_pad=50304, batch=8, lr=1e-4,
                  zipf=1.1, preset="aggressive", preset_levels=True),
}


def build_gpt(torch, nn, F, apa, cfgd, device):
    from apa import APAConfig, APALinear
    preset = {"default": APAConfig, "aggressive": APAConfig.aggressive}[cfgd["preset"]]
    cfg = preset(device=str(device)) if cfgd["preset"] != "default" else APAConfig(device=str(device))
    d, H, T = cfgd["d"], cfgd["n_head"], cfgd["T"]

    class LayerNorm32(nn.LayerNorm):
        """LayerNorm in fp32 that accepts the fp16 outputs of FP16-rung layers
        and returns fp32 (the residual stream's dtype)."""

        def forward(self, x):
            return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps)

    class Attention(nn.Module):
        def __init__(self):
            super().__init__()
            self.c_attn = APALinear(d, 3 * d, config=cfg)
            self.c_proj = APALinear(d, d, config=cfg)

        def forward(self, x):
            B, Tq, C = x.shape
            q, k, v = self.c_attn(x).to(torch.bfloat16).split(C, dim=2)
            q = q.view(B, Tq, H, C // H).transpose(1, 2)
            k = k.view(B, Tq, H, C // H).transpose(1, 2)
            v = v.view(B, Tq, H, C // H).transpose(1, 2)
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            return self.c_proj(y.transpose(1, 2).reshape(B, Tq, C))

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.c_fc = APALinear(d, 4 * d, config=cfg)
            self.gelu = nn.GELU()
            self.c_proj = APALinear(4 * d, d, config=cfg)

        def forward(self, x):
            return self.c_proj(self.gelu(self.c_fc(x).float()))

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln_1 = LayerNorm32(d)
            self.attn = Attention()
            self.ln_2 = LayerNorm32(d)
            self.mlp = MLP()

        def forward(self, x):
            x = x + self.attn(self.ln_1(x)).float()
            return x + self.mlp(self.ln_2(x)).float()

    class GPT(nn.Module):
        def __init__(self):
            super().__init__()
            self.token_embedding = nn.Embedding(cfgd["vocab"], d)
            self.position_embedding = nn.Embedding(T, d)
            self.blocks = nn.ModuleList([Block() for _ in range(cfgd["n_layer"])])
            self.ln_f = LayerNorm32(d)
            self.lm_head = APALinear(d, cfgd["vocab_pad"], config=cfg)

        def forward(self, idx):
            B, Tq = idx.shape
            pos = torch.arange(Tq, device=idx.device)
            x = self.token_embedding(idx) + self.position_embedding(pos)
            for blk in self.blocks:
                x = blk(x)
            return self.lm_head(self.ln_f(x))

    torch.manual_seed(0)
    model = GPT().to(device)
    if cfgd["preset_levels"]:
        for i in range(4):
            model.blocks[i].attn.c_attn.level = 1
        model.lm_head.level = 2
    if cfgd["vocab_pad"] > cfgd["vocab"]:
        assert model.lm_head.level == 2, "padded classes need an fp32 bias"
        with torch.no_grad():
            model.lm_head.bias_master[cfgd["vocab"]:] = -30000.0
    return model, cfg


def gpt_batches(torch, cfgd, rank, device, n=4):
    g = torch.Generator().manual_seed(1234 + rank)
    B, T, V = cfgd["batch"], cfgd["T"], cfgd["vocab"]
    out = []
    for _ in range(n):
        if cfgd["zipf"]:
            ranks = torch.arange(1, V + 1, dtype=torch.float64)
            p = ranks.pow(-cfgd["zipf"])
            idx = torch.multinomial(p / p.sum(), B * (T + 1), replacement=True, generator=g)
        else:
            idx = torch.randint(0, V, (B * (T + 1),), generator=g)
        idx = idx.view(B, T + 1)
        out.append((idx[:, :T].contiguous().to(device), idx[:, 1:].contiguous().to(device)))
    return out


def run_gpt(torch, dist, name, world, rank, dev, steps, warmup, barrier, max_over_ranks, graphed=True,
            optimizer="torch", dp_block_bytes=0, dp_bucket_bytes=64 << 20, dp_nvls=True):
    import torch.nn as nn
    import torch.nn.functional as F
    import apa
    from apa import APAManager
    cfgd = GPT_CONFIGS[name]
    model, cfg = build_gpt(torch, nn, F, apa, cfgd, dev)
    mgr = APAManager(model, cfg, bucket_bytes=dp_bucket_bytes, dp_block_bytes=dp_block_bytes, dp_nvls=dp_nvls)
    if optimizer == "apa":
        # AdamW with each APALinear weight's next working copy written in the same pass
        from apa.optim import APAAdamW
        opt = APAAdamW(mgr, lr=cfgd["lr"], weight_decay=0.01)
    else:
        opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=cfgd["lr"], weight_decay=0.01, fused=True)
    batches = gpt_batches(torch, cfgd, rank, dev)
    V = cfgd["vocab_pad"]

    def loss_fn(x, y):
        return F.cross_entropy(model(x).reshape(-1, V).float(), y.reshape(-1))

    if graphed:
        from apa.graphs import GraphedTrainStep
        gstep = GraphedTrainStep(mgr, loss_fn, batches[0], warmup=2)

        def step(i):
            loss, keep = gstep(*batches[i % len(batches)])
            if keep:
                opt.step()
            return loss
    else:
        def step(i):
            x, y = batches[i % len(batches)]
            mgr.pre_step()
            opt.zero_grad(set_to_none=True)
            loss = loss_fn(x, y)
            loss.backward()
            if mgr.post_backward_sync_and_eval():
                opt.step()
            else:
                opt.zero_grad(set_to_none=True)
            return loss

    for i in range(warmup):
        step(i)
    barrier()
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        loss = step(warmup + i)
    e1.record(s)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    tokens = world * cfgd["batch"] * cfgd["T"]
    nparam = sum(m.weight_master.numel() for m in mgr.apa_modules.values())
    levels = {}
    for m in mgr.apa_modules.values():
        levels[m.level] = levels.get(m.level, 0) + 1
    out = {"tokens_per_s": round(tokens / ms * 1e3, 1), "ms_per_step": round(ms, 3), "global_batch_tokens": tokens,
           "mode": "cuda-graph replay of pre_step+fwd+bwd" if graphed else "eager",
           "optimizer": "APAAdamW (fused weight update + working-copy cast)" if optimizer == "apa"
           else "torch.optim.AdamW(fused=True)",
           "apa_linear_params": nparam, "levels": {["fp8", "fp16", "tf32"][k]: v for k, v in sorted(levels.items())},
           "loss": round(float(loss.item()), 4)}
    del model, mgr, opt
    torch.cuda.empty_cache()
    return out


# ViT classifier on 32x32x3 images: patch 4 (48-wide patch embedding, 64
# patches + a class token = 65 tokens), d 512, depth 6, 8 heads, MLP 1024, 10
# classes, APALinear for the patch embedding, QKV, projection, MLP and head;
# per-GPU batch 512, pixels ~ N(0,1), uniform labels, conservative() config.
VIT_CONFIG = dict(img=32, patch=4, ch=3, d=512, depth=6, heads=8, mlp=1024, classes=10, batch=512, lr=1e-3)


def build_vit(torch, nn, F, apa, cfgd, device):
    from apa import APAConfig, APALinear
    cfg = APAConfig.conservative(device=str(device))
    d, H, P = cfgd["d"], cfgd["heads"], cfgd["patch"]
    n_patch = (cfgd["img"] // P) ** 2
    pdim = cfgd["ch"] * P * P

    class LayerNorm32(nn.LayerNorm):
        def forward(self, x):
            return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.norm1 = LayerNorm32(d)
            self.qkv = APALinear(d, 3 * d, config=cfg)
            self.out_proj = APALinear(d, d, config=cfg)
            self.norm2 = LayerNorm32(d)
            self.mlp = nn.Sequential(APALinear(d, cfgd["mlp"], config=cfg), nn.GELU(),
                                     APALinear(cfgd["mlp"], d, config=cfg))

        def forward(self, x):
            B, T, C = x.shape
            q, k, v = self.qkv(self.norm1(x)).to(torch.bfloat16).split(C, dim=2)
            q, k, v = (t.view(B, T, H, C // H).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v)
            x = x + self.out_proj(a.transpose(1, 2).reshape(B, T, C)).float()
            return x + self.mlp(self.norm2(x)).float()

    class ViT(nn.Module):
        def __init__(self):
            super().__init__()
            self.patch_embed = APALinear(pdim, d, config=cfg)
            self.cls_token = nn.Parameter(torch.zeros(1, 1, d))
            self.pos_embed = nn.Parameter(torch.randn(1, n_patch + 1, d) * 0.02)
            self.blocks = nn.ModuleList([Block() for _ in range(cfgd["depth"])])
            self.norm = LayerNorm32(d)
            self.head = APALinear(d, cfgd["classes"], config=cfg)

        def forward(self, img):
            B = img.shape[0]
            g = cfgd["img"] // P
            patches = img.view(B, cfgd["ch"], g, P, g, P).permute(0, 2, 4, 1, 3, 5).reshape(B, g * g, pdim)
            x = self.patch_embed(patches).float()
            x = torch.cat([self.cls_token.expand(B, -1, -1), x], dim=1) + self.pos_embed
            for blk in self.blocks:
                x = blk(x)
            return self.head(self.norm(x[:, 0]))

    torch.manual_seed(0)
    return ViT().to(device), cfg


def run_vit(torch, world, rank, dev, steps, warmup, barrier, max_over_ranks, graphed=True, dp_bucket_bytes=64 << 20,
            dp_nvls=True):
    import torch.nn as nn
    import torch.nn.functional as F
    import apa
    from apa import APAManager
    cfgd = VIT_CONFIG
    model, cfg = build_vit(torch, nn, F, apa, cfgd, dev)
    mgr = APAManager(model, cfg, bucket_bytes=dp_bucket_bytes, dp_nvls=dp_nvls)
    opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=cfgd["lr"], weight_decay=0.01, fused=True)
    g = torch.Generator().manual_seed(4321 + rank)
    B = cfgd["batch"]
    batches = [(torch.randn(B, cfgd["ch"], cfgd["img"], cfgd["img"], generator=g).to(dev),
                torch.randint(0, cfgd["classes"], (B,), generator=g).to(dev)) for _ in range(4)]

    def loss_fn(x, y):
        return F.cross_entropy(model(x).float(), y)

    if graphed:
        from apa.graphs import GraphedTrainStep
        gstep = GraphedTrainStep(mgr, loss_fn, batches[0], warmup=2)

        def step(i):
            loss, keep = gstep(*batches[i % len(batches)])
            if keep:
                opt.step()
            return loss
    else:
        def step(i):
            x, y = batches[i % len(batches)]
            mgr.pre_step()
            opt.zero_grad(set_to_none=True)
            loss = loss_fn(x, y)
            loss.backward()
            if mgr.post_backward_sync_and_eval():
                opt.step()
            return loss

    for i in range(warmup):
        step(i)
    barrier()
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        loss = step(warmup + i)
    e1.record(s)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    images = world * B
    levels = {}
    for m in mgr.apa_modules.values():
        levels[m.level] = levels.get(m.level, 0) + 1
    out = {"images_per_s": round(images / ms * 1e3, 1), "ms_per_step": round(ms, 3), "global_batch_images": images,
           "mode": "cuda-graph replay of pre_step+fwd+bwd" if graphed else "eager",
           "optimizer": "torch.optim.AdamW(fused=True)",
           "apa_linear_params": sum(m.weight_master.numel() for m in mgr.apa_modules.values()),
           "levels": {["fp8", "fp16", "tf32"][k]: v for k, v in sorted(levels.items())},
           "loss": round(float(loss.item()), 4)}
    gstep = None
    del model, mgr, opt
    torch.cuda.empty_cache()
    return out


def time_gemm(torch, _lib, lin, xr, dev, pk, libpk):
    """The dominant kernel: the FP8 tcgen05 GEMM (forward, 8192x4096x4096),
    timed alone with CUDA events on its launching stream. Also times the same
    GEMM without bias twice, with the fused telemetry (amax / NaN flag of y)
    and bare (apa_gemm_tn: no telemetry work at all), for the telemetry cost."""
    lib = _lib.lib()
    wq = lin._wq
    xq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev)
    _lib.check(lib.apa_cast(xr.data_ptr(), _lib.DT_BF16, M, K, K, xq.data_ptr(), _lib.DT_E4M3, K, None, 0,
                            None, None, 0, None, None, _lib.stream_handle(dev)), "cast")
    y = torch.empty(M, N, device=dev)
    amax = torch.zeros(1, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    st = _lib.stream_handle(dev)

    def fused(bias):
        _lib.check(lib.apa_linear_fwd(0, xq.data_ptr(), K, wq.data_ptr(), wq.stride(0), bias, y.data_ptr(), N, M, N,
                                      K, amax.data_ptr(), flag.data_ptr(), st), "fwd")

    def bare():
        _lib.check(lib.apa_gemm_tn(0, 0, xq.data_ptr(), K, wq.data_ptr(), wq.stride(0), y.data_ptr(), _lib.DT_F32, N,
                                   M, N, K, 0, 0, st), "gemm_tn")

    def timed(fn, reps=50):
        for _ in range(5):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    us = timed(lambda: fused(lin._bq.data_ptr()))
    # sustained: the same launch back to back for ~0.4 s with the SM clock
    # sampled meanwhile; under this load the 1000 W cap holds the clock well
    # below its 1965 MHz maximum, so the tensor pipe's peak at the clock the
    # kernel actually ran at (148 SMs x 16384 dense FP8 FLOP per clock) is the
    # denominator that separates kernel efficiency from the power cap
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.__enter__()
    us_sus = timed(lambda: fused(lin._bq.data_ptr()), 4000)
    sampler.__exit__()
    clk = sampler.summary()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    clock_peak = sms * 16384 * clk["sm_mhz"] * 1e6 / 1e12 if clk.get("sm_mhz") else None
    # alternate the two telemetry variants so clock drift affects both alike
    t_tel, t_bare = [], []
    for _ in range(3):
        t_tel.append(timed(lambda: fused(None), 30))
        t_bare.append(timed(bare, 30))
    tel, bar = min(t_tel), min(t_bare)
    achieved = 2.0 * M * N * K / (us * 1e-6) / 1e12
    lib_fp8 = libpk.get("fp8_tflops")
    tile, ew = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.apa_gemm_plan(0, 0, M, N, K, _lib.DT_F32, 0, 0, ctypes.addressof(tile), ctypes.addressof(ew)),
               "plan")
    shape = {128: "128x128", 256: "128x256", 512: "256x256 CTA pair"}[tile.value]
    return {"kernel": f"gemm_kernel E4M3 forward 8192x4096x4096, {shape} tile, {ew.value} epilogue warps",
            "bound": "tensor",
            "achieved": round(achieved, 1), "peak": pk["fp8_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["fp8_tflops"], 4), "us_per_launch": round(us, 2),
            "frac_of_spec_fp8": round(achieved / 4500.0, 4),
            "sustained": {"us_per_launch": round(us_sus, 2), "launches": 4000, "sm_mhz": clk.get("sm_mhz"),
                          "reasons": clk.get("reasons"),
                          "achieved": round(2.0 * M * N * K / (us_sus * 1e-6) / 1e12, 1),
                          "tensor_peak_at_clock": round(clock_peak, 1) if clock_peak else None,
                          "frac_of_peak_at_clock": round(2.0 * M * N * K / (us_sus * 1e-6) / 1e12 / clock_peak, 4)
                          if clock_peak else None},
            "frac_of_library_fp8": round(achieved / lib_fp8, 4) if lib_fp8 else None,
            "peak_note": f"2 x {pk['source']} bf16 cuBLAS burst ({pk['bf16_tflops']} TFLOP/s); "
                         "frac_of_spec_fp8 is against the 4500 TFLOP/s dense FP8 specification",
            "telemetry": {"us_with": round(tel, 2), "us_bare": round(bar, 2),
                          "overhead": round(tel / bar - 1.0, 4),
                          "note": "forward without bias: fused amax/NaN telemetry vs the same kernel with none"},
            # dram__bytes_read.sum + dram__bytes_write.sum of this kernel from one ncu
            # capture (profiles/gemm_fp8_fwd_8192x4096x4096.md), bytes per launch
            "traffic": 145.9e6}


def time_optimizer(torch, _lib, dev, pk):
    """AdamW on the 4096x4096 master weight fused with its next FP8 working
    copies (apa_adamw_cast: p, m, v updated, W_q and W_q^T written, weight
    amax), against torch.optim.AdamW(fused=True) followed by the library's
    cast of the updated weight. CUDA events on the launching stream; every
    launch streams about 0.5 GB, four times the L2."""
    lib = _lib.lib()
    st = _lib.stream_handle(dev)
    s = torch.cuda.current_stream(dev)
    g0 = torch.Generator(device=dev).manual_seed(5)
    p = torch.randn(N, K, device=dev, generator=g0) * 0.02
    g = torch.randn(N, K, device=dev, generator=g0) * 1e-3
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    wq = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=dev)
    wqt = torch.empty(K, N, dtype=torch.float8_e4m3fn, device=dev)
    amax = torch.zeros(1, device=dev)
    pt = p.clone().requires_grad_(True)
    pt.grad = g.clone()
    opt = torch.optim.AdamW([pt], lr=1e-3, weight_decay=0.01, fused=True)
    n = [0]

    def fused():
        n[0] += 1
        _lib.check(lib.apa_adamw_cast(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), N, K, K, 1e-3, 0.9,
                                      0.999, 1e-8, 0.01, n[0], wq.data_ptr(), _lib.DT_E4M3, K, wqt.data_ptr(), N,
                                      amax.data_ptr(), st), "adamw_cast")

    def separate():
        opt.step()
        _lib.check(lib.apa_cast(pt.data_ptr(), _lib.DT_F32, N, K, K, wq.data_ptr(), _lib.DT_E4M3, K, wqt.data_ptr(),
                                N, amax.data_ptr(), None, 0, None, None, st), "cast")

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    t_f, t_s = [], []
    for _ in range(2):
        t_f.append(timed(fused))
        t_s.append(timed(separate))
    tf, ts = min(t_f), min(t_s)
    # algorithmic bytes: read p, g, m, v (fp32), write p, m, v (fp32) and the two E4M3 copies
    nbytes = N * K * (7 * 4 + 2)
    gbs = nbytes / (tf * 1e-6) / 1e9
    return {"kernel": "adamw_cast_kernel E4M3, 4096x4096 fp32 master", "bound": "hbm",
            "us_per_launch": round(tf, 2), "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(gbs / pk["hbm_gbs"], 4), "bytes_per_launch": nbytes,
            "torch_adamw_fused_plus_cast_us": round(ts, 2), "speedup": round(ts / tf, 3)}


def run_e2e(torch, make, x, dy32, dev, args, world, barrier, max_over_ranks):
    """End to end through the public API with host-resident inputs: every
    step's x and dy are copied from pinned host memory and the step's decision
    record is read back. The copies of step i+1 run on a copy stream while
    step i computes (two device buffer sets); the timed region starts before
    the first copy is issued and ends after the last step, so it holds every
    step's copies and computations."""
    lin, mgr = make(0)
    xh = x.cpu().pin_memory()
    dyh = dy32.cpu().pin_memory()
    xd = [torch.empty_like(x), torch.empty_like(x)]
    dyd = [torch.empty_like(dy32), torch.empty_like(dy32)]
    cur = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    used = [torch.cuda.Event(), torch.cuda.Event()]
    for k in range(2):
        used[k].record(cur)

    def issue_copy(k):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(used[k])          # the step that read set k is done
            xd[k].copy_(xh, non_blocking=True)
            dyd[k].copy_(dyh, non_blocking=True)
            copied[k].record(copy_stream)

    def step(i, n):
        k = i % 2
        cur.wait_event(copied[k])
        xr = xd[k].requires_grad_(True)
        mgr.pre_step()
        lin(xr).backward(dyd[k])
        ok = mgr.post_backward_sync_and_eval()    # reads the step's decision record back
        xr.grad = None
        xr.requires_grad_(False)
        used[k].record(cur)
        if i + 2 < n:
            issue_copy(k)                         # inputs of step i + 2
        return ok

    def run(n, timed):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        copy_stream.wait_event(e0)
        for k in range(min(2, n)):
            issue_copy(k)
        for i in range(n):
            step(i, n)
        e1.record(cur)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    run(max(2, args.warmup), False)
    barrier()
    steps = max(3, args.steps // 2)
    ms = max_over_ranks(run(steps, True) / steps)
    rec_bytes = mgr._ladder.nbytes
    return {"value": round(world * FLOPS_STEP / ms / 1e9, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": int(x.numel() * x.element_size() + dy32.numel() * 4),
            "d2h_bytes_per_step": int(rec_bytes),
            "api": "APAManager.pre_step / APALinear fwd+bwd / post_backward_sync_and_eval, pinned host inputs, "
                   "next step's copies overlapped with the current step"}


# ---------------------------------------------------------------------------
# the reference's CPU path
# ---------------------------------------------------------------------------
def reference_impl():
    """The reference's CPU implementation of the path, as (kind, module):
    the reference package itself when it is installed under baseline/_ref
    ("reference"), else the torch-CPU port of its fp8_simulation_mode path
    (oracle/ref_port.py, "port"), which reproduces the reference's outputs,
    telemetry and cfg0 trajectory bit for bit (tests/test_ref_port_cpu.py)
    with the same torch operations, so it costs what the reference costs."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(os.path.join(ref, "apa")):
        for k in [k for k in sys.modules if k == "apa" or k.startswith("apa.")]:
            del sys.modules[k]
        sys.path.insert(0, ref)
        try:
            import apa as ref_apa
        finally:
            sys.path.remove(ref)
        if os.path.abspath(ref_apa.__file__).startswith(os.path.abspath(ref)):
            return "reference", ref_apa
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import ref_port
    return "port", ref_port


def ref_step_fn(kind, mod, torch, level=0):
    """One cfg1 training step (pre_step, forward, backward, evaluation) of the
    reference's CPU path at the full 8192x4096x4096 shape, same seeds as the
    GPU arm: layer initialised under torch.manual_seed(0), x bf16 N(0,1) from
    a CPU generator seeded 0, dy N(0,1) seeded 1 (fp16 at the FP16 rung)."""
    import torch.nn as nn
    torch.manual_seed(0)
    if kind == "reference":
        cfg = mod.APAConfig(fp8_simulation_mode=True, device="cpu", check_interval=1)
        lin = mod.APALinear(K, N, config=cfg)
        mgr = mod.APAManager(nn.Sequential(lin), cfg)
    else:
        lin = mod.PortLinear(K, N)
        mgr = mod.PortManager(nn.Sequential(lin), check_interval=1)
    lin.level = level
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(M, N, generator=torch.Generator().manual_seed(1))
    if level == 1:
        dy = dy.half()

    def step():
        mgr.pre_step()
        lin(x).backward(dy)
        x.grad = None
        return mgr.post_backward_sync_and_eval()
    return step


CFG0_STEPS = 200
CFG0_SPIKES = (50, 150)


def cfg0_inputs(torch):
    """cfg0's seeded batch: x [64, 768] N(0,1) and labels in [0, 10) from a
    CPU generator seeded 0, then for each spike step (50 and 150, 0-based)
    49 element indices (0.1 %) whose values are scaled by 1e3 on that step."""
    g = torch.Generator().manual_seed(0)
    x0 = torch.randn(64, 768, generator=g)
    y0 = torch.randint(0, 10, (64,), generator=g)
    spikes = {s: torch.randperm(x0.numel(), generator=g)[:49] for s in CFG0_SPIKES}
    return x0, y0, spikes


def cfg0_cpu(kind, mod, torch):
    """cfg0 (APALinear(768,768) -> ReLU -> LayerNorm(768) -> APALinear(768,10),
    AdamW 1e-3, research_default, batch 64, 200 steps with two input spikes)
    on the reference's CPU path: steps/s over the 200 steps."""
    import torch.nn as nn
    import torch.nn.functional as F
    torch.manual_seed(0)
    if kind == "reference":
        cfg = mod.APAConfig.research_default(fp8_simulation_mode=True, device="cpu")
        lin = lambda i, o: mod.APALinear(i, o, config=cfg)
    else:
        lin = mod.PortLinear
    model = nn.Sequential(lin(768, 768), nn.ReLU(), nn.LayerNorm(768), lin(768, 10))
    if kind == "reference":
        mgr = mod.APAManager(model, cfg)
        params = mgr.get_trainable_parameters()
    else:
        mgr = mod.PortManager(model, theta=0.40, alpha=0.95, check_interval=4)
        params = mgr.trainable()
    opt = torch.optim.AdamW(params, lr=1e-3)
    x0, y0, spikes = cfg0_inputs(torch)
    skips = []
    t0 = time.perf_counter()
    for step in range(CFG0_STEPS):
        x = x0.clone()
        if step in spikes:
            x.view(-1)[spikes[step]] *= 1e3
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(model(x), y0).backward()
        if mgr.post_backward_sync_and_eval():
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
            skips.append(step)
    dt = time.perf_counter() - t0
    return {"steps_per_s": round(CFG0_STEPS / dt, 2), "steps": CFG0_STEPS, "skipped_steps": skips,
            "cores": torch.get_num_threads(), "kind": kind}


def cfg0_gpu(torch, dev):
    """cfg0 through this library's API on the GPU (same model, seeds, spikes
    and optimizer as cfg0_cpu): steps/s over the 200 steps, each step ending
    in the ladder's host read, timed with CUDA events on the current stream."""
    import torch.nn as nn
    import torch.nn.functional as F
    from apa import APAConfig, APALinear, APAManager
    cfg = APAConfig.research_default(device=str(dev))

    class MixedLayerNorm(nn.LayerNorm):
        # accepts the fp16 output of an FP16-rung layer (torch's CPU LayerNorm
        # does, its CUDA one does not) and returns the input's dtype
        def forward(self, x):
            return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps).to(x.dtype)

    torch.manual_seed(0)
    model = nn.Sequential(APALinear(768, 768, config=cfg), nn.ReLU(), MixedLayerNorm(768),
                          APALinear(768, 10, config=cfg)).to(dev)
    mgr = APAManager(model, cfg)
    opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=1e-3)
    x0, y0, spikes = cfg0_inputs(torch)
    x0, y0 = x0.to(dev), y0.to(dev)
    spikes = {k: v.to(dev) for k, v in spikes.items()}
    skips = []
    s = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for step in range(CFG0_STEPS):
        x = x0.clone()
        if step in spikes:
            x.view(-1)[spikes[step]] *= 1e3
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(model(x), y0).backward()
        if mgr.post_backward_sync_and_eval():
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
            skips.append(step)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    return {"steps_per_s": round(CFG0_STEPS / ms * 1e3, 2), "steps": CFG0_STEPS, "skipped_steps": skips,
            "mode": "eager, one host read per step"}


def _quiet(fn, *a):
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):   # the reference's event logger prints
        return fn(*a)


def cpu_baseline(args, sample_steps=1):
    import torch
    kind, mod = reference_impl()
    torch.set_num_threads(os.cpu_count())
    step = ref_step_fn(kind, mod, torch)

    def run():
        step()
        t0 = time.perf_counter()
        for _ in range(sample_steps):
            step()
        return (time.perf_counter() - t0) / sample_steps
    dt = _quiet(run)
    src = ("the reference's fp8_simulation_mode CPU path" if kind == "reference" else
           "the torch-CPU port of the reference's fp8_simulation_mode path (oracle/ref_port.py)")
    return {"value": round(FLOPS_STEP / dt / 1e12, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": kind,
            "sample": f"{src}, FP8 rung, full 8192x4096x4096 step, {sample_steps} timed step(s) after 1 warm-up, "
                      f"{dt:.2f} s/step, torch {torch.__version__}"}


def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path on
    this host's cores (all of them), FP8 rung at the full cfg1 shape, each
    step a full training step; at most 10 timed steps after at most 2 warm-up
    steps so the run stays within about a minute. Rank 0 only under torchrun."""
    world, rank, _ = dist_info()
    if rank != 0:
        return None
    import torch
    kind, mod = reference_impl()
    torch.set_num_threads(os.cpu_count())
    step = ref_step_fn(kind, mod, torch)
    steps = max(1, min(args.steps, 10))
    warm = max(1, min(args.warmup, 2))

    def run():
        for _ in range(warm):
            step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        return (time.perf_counter() - t0) / steps
    dt = _quiet(run)
    cfg0 = _quiet(cfg0_cpu, kind, mod, torch)
    v = round(FLOPS_STEP / dt / 1e12, 4)
    src = ("the reference's fp8_simulation_mode CPU path (baseline/_ref)" if kind == "reference" else
           "the torch-CPU port of the reference's fp8_simulation_mode path (oracle/ref_port.py; the reference "
           "package is not installed here)")
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
            "config": dict(CONFIG, parallelism="cpu"),
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": kind,
                             "sample": f"{src}, FP8 rung, {steps} full 8192x4096x4096 steps (of the requested "
                                       f"{args.steps}) after {warm} warm-up, torch {torch.__version__}"},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "cfg0": cfg0}


def gemm_table():
    """FP8 GEMMs of the GPT-2-medium layers (8192 tokens, d 1024, MLP 4096),
    each timed back to back: a CUDA graph of 12 launches replayed, CUDA events
    around one replay, the best of 5 (microseconds per launch, including the
    2-4 us between consecutive kernels). Columns: the layer's fused entry
    point (forward with bias and telemetry; input gradient with fp32 dx and
    boundary-cast telemetry; weight gradient with counts and its split
    workspace), the same GEMM bare (apa_gemm_tn, raw fp32 accumulator), and
    cuBLASLt FP8 (torch._scaled_mm, unit scales, fp32 output) on the same
    operands. One JSON line per GEMM."""
    sys.path.insert(0, PKG)
    import torch
    from apa import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    e4 = torch.float8_e4m3fn
    T, NL = 8192, 12
    one = torch.ones((), device=dev)

    def per_launch(fn):
        fn()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(NL):
                fn()
        for _ in range(3):
            graph.replay()
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / NL
            best = us if best is None else min(best, us)
        del graph
        return round(best, 2)

    amax = torch.zeros(1, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    layers = {"qkv": (3072, 1024), "proj": (1024, 1024), "fc": (4096, 1024), "fc2": (1024, 4096)}
    for name, (nout, nin) in layers.items():
        x = torch.randn(T, nin, device=dev, generator=g).to(e4)
        w = (torch.randn(nout, nin, device=dev, generator=g) * 0.05).to(e4)
        b = (torch.randn(nout, device=dev, generator=g) * 0.1).to(e4)
        dy = torch.randn(T, nout, device=dev, generator=g).to(e4)
        wt, dyt, xt = w.t().contiguous(), dy.t().contiguous(), x.t().contiguous()
        for op in ("fwd", "dgrad", "wgrad"):
            if op == "fwd":
                A, B, m, n, k = x, w, T, nout, nin
                out = torch.empty(m, n, device=dev)

                def fused():
                    _lib.check(lib.apa_linear_fwd(0, x.data_ptr(), nin, w.data_ptr(), nin, b.data_ptr(),
                                                  out.data_ptr(), nout, T, nout, nin, amax.data_ptr(),
                                                  flag.data_ptr(), _lib.stream_handle(dev)), "fwd")
            elif op == "dgrad":
                A, B, m, n, k = dy, wt, T, nin, nout
                out = torch.empty(m, n, device=dev)

                def fused():
                    _lib.check(lib.apa_linear_dgrad(0, dy.data_ptr(), nout, wt.data_ptr(), nout, out.data_ptr(),
                                                    _lib.DT_F32, nin, T, nout, nin, amax.data_ptr(), flag.data_ptr(),
                                                    _lib.stream_handle(dev)), "dgrad")
            else:
                A, B, m, n, k = dyt, xt, nout, nin, T
                out = torch.empty(m, n, device=dev)
                cnt = torch.zeros(3, dtype=torch.int64, device=dev)
                nb = ctypes.c_int64(0)
                _lib.check(lib.apa_wgrad_workspace_bytes(0, T, nout, nin, ctypes.addressof(nb)), "ws")
                ws = torch.empty(max(nb.value, 16), dtype=torch.uint8, device=dev)

                def fused():
                    if nb.value > 0:
                        _lib.check(lib.apa_linear_wgrad_ws(0, dyt.data_ptr(), T, xt.data_ptr(), T, out.data_ptr(), nin,
                                                           T, nout, nin, 0, cnt.data_ptr(), amax.data_ptr(),
                                                           ws.data_ptr(), nb.value, _lib.stream_handle(dev)), "wgrad")
                    else:
                        _lib.check(lib.apa_linear_wgrad(0, dyt.data_ptr(), T, xt.data_ptr(), T, out.data_ptr(), nin,
                                                        T, nout, nin, 0, cnt.data_ptr(), amax.data_ptr(),
                                                        _lib.stream_handle(dev)), "wgrad")
            raw = torch.empty(m, n, device=dev)

            def bare():
                _lib.check(lib.apa_gemm_tn(0, 3, A.data_ptr(), k, B.data_ptr(), k, raw.data_ptr(), _lib.DT_F32, n, m,
                                           n, k, 0, 0, _lib.stream_handle(dev)), "gemm_tn")

            def cublas():
                torch._scaled_mm(A, B.t(), scale_a=one, scale_b=one, out_dtype=torch.float32)

            tile, ew = ctypes.c_int(0), ctypes.c_int(0)
            _lib.check(lib.apa_gemm_plan(0, {"fwd": 0, "dgrad": 1, "wgrad": 2}[op], m, n, k, _lib.DT_F32, 0, 0,
                                         ctypes.addressof(tile), ctypes.addressof(ew)), "plan")
            row = {"gemm": f"{name} {op}", "M": m, "N": n, "K": k, "plan": [tile.value, ew.value],
                   "fused_us": per_launch(fused), "bare_us": per_launch(bare)}
            try:
                row["cublaslt_us"] = per_launch(cublas)
            except RuntimeError as e:
                row["cublaslt_us"] = None
                row["cublaslt_error"] = str(e)[:120]
            row["tflops_fused"] = round(2.0 * m * n * k / (row["fused_us"] * 1e-6) / 1e12, 1)
            print(json.dumps(row), flush=True)


def profile_case(case: str):
    """A few launches of one kernel at the bench shape, for ncu captures:
    gemm-fp8 / gemm-fp16 / gemm-tf32 (forward GEMM), dgrad-<rung> and
    wgrad-<rung> (input / weight gradient GEMMs), cast (bf16 x -> E4M3 and its
    transposed copy), dyprep (fp32 dy -> E4M3 + transposed + bias partials),
    cast-tf32 / dyprep-tf32 (the same at the TF32 rung), adamw-fp8, and
    one-step launch lists (step-*)."""
    sys.path.insert(0, PKG)
    import torch
    from apa import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    st = _lib.stream_handle(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    if case == "gemm-fp8-k1024":
        # an epilogue-bound FP8 forward: GPT-2-medium attention QKV projection
        # (8192 tokens, 1024 -> 3072), fp32 output with bias and telemetry
        Mq, Kq, Nq = 8192, 1024, 3072
        x = torch.randn(Mq, Kq, device=dev, generator=g).to(torch.float8_e4m3fn)
        w = (torch.randn(Nq, Kq, device=dev, generator=g) * 0.02).to(torch.float8_e4m3fn)
        b = (torch.randn(Nq, device=dev, generator=g) * 0.1).to(torch.float8_e4m3fn)
        y = torch.empty(Mq, Nq, device=dev)
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(3):
            _lib.check(lib.apa_linear_fwd(0, x.data_ptr(), Kq, w.data_ptr(), Kq, b.data_ptr(), y.data_ptr(), Nq, Mq,
                                          Nq, Kq, amax.data_ptr(), flag.data_ptr(), st), "fwd")
    elif case.startswith("gemm"):
        rung = {"gemm-fp8": 0, "gemm-fp16": 1, "gemm-tf32": 2}[case]
        dt = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}[rung]
        x = torch.randn(M, K, device=dev, generator=g).to(dt)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(dt)
        y = torch.empty(M, N, device=dev, dtype=torch.float16 if rung == 1 else torch.float32)
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(3):
            _lib.check(lib.apa_linear_fwd(rung, x.data_ptr(), K, w.data_ptr(), K, None, y.data_ptr(), N, M, N, K,
                                          amax.data_ptr(), flag.data_ptr(), st), "fwd")
    elif case.split("-")[0] in ("dgrad", "wgrad"):
        # input / weight gradient GEMM at the bench shape with its fused
        # epilogue: dx bf16 with boundary-cast telemetry, or dw fp32 with the
        # underflow counts and ratio fold
        op, rname = case.split("-")
        rung = {"fp8": 0, "fp16": 1, "tf32": 2}[rname]
        dt = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}[rung]
        dyq = torch.randn(M, N, device=dev, generator=g).to(dt)
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        if op == "dgrad":
            wqt = (torch.randn(K, N, device=dev, generator=g) * 0.02).to(dt)
            dx = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
            for _ in range(3):
                _lib.check(lib.apa_linear_dgrad(rung, dyq.data_ptr(), N, wqt.data_ptr(), N, dx.data_ptr(),
                                                _lib.DT_BF16, K, M, N, K, amax.data_ptr(), flag.data_ptr(), st),
                           "dgrad")
        else:
            dyqt = dyq.t().contiguous()
            xqt = torch.randn(K, M, device=dev, generator=g).to(dt)
            dw = torch.empty(N, K, device=dev)
            cnt = torch.zeros(3, dtype=torch.int64, device=dev)
            for _ in range(3):
                _lib.check(lib.apa_linear_wgrad(rung, dyqt.data_ptr(), M, xqt.data_ptr(), M, dw.data_ptr(), K, M, N,
                                                K, 0, cnt.data_ptr(), amax.data_ptr(), st), "wgrad")
    elif case in ("cast-tf32", "dyprep-tf32"):
        # the TF32 rung's casts: x bf16 -> TF32-rounded fp32 and its transposed
        # copy; dy fp32 -> TF32 + transposed + bias partial sums
        src_dt, code = (torch.bfloat16, _lib.DT_BF16) if case == "cast-tf32" else (torch.float32, _lib.DT_F32)
        src = torch.randn(M, K, device=dev, generator=g).to(src_dt)
        q = torch.empty(M, K, device=dev)
        qt = torch.empty(K, M, device=dev)
        part = torch.empty(M // 64, K, device=dev) if case == "dyprep-tf32" else None
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(3):
            _lib.check(lib.apa_cast(src.data_ptr(), code, M, K, K, q.data_ptr(), _lib.DT_TF32, K, qt.data_ptr(), M,
                                    amax.data_ptr(), flag.data_ptr(), 1 if part is not None else 0, None,
                                    _lib.ptr(part), st), case)
    elif case == "cast":
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        xq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev)
        xqt = torch.empty(K, M, dtype=torch.float8_e4m3fn, device=dev)
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(3):
            _lib.check(lib.apa_cast(x.data_ptr(), _lib.DT_BF16, M, K, K, xq.data_ptr(), _lib.DT_E4M3, K,
                                    xqt.data_ptr(), M, amax.data_ptr(), flag.data_ptr(), 0, None, None, st), "cast")
    elif case == "dyprep":
        dy = torch.randn(M, N, device=dev, generator=g)
        dq = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=dev)
        dqt = torch.empty(N, M, dtype=torch.float8_e4m3fn, device=dev)
        part = torch.empty(M // 64, N, device=dev)
        amax = torch.zeros(1, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(3):
            _lib.check(lib.apa_cast(dy.data_ptr(), _lib.DT_F32, M, N, N, dq.data_ptr(), _lib.DT_E4M3, N,
                                    dqt.data_ptr(), M, amax.data_ptr(), flag.data_ptr(), 1, None, part.data_ptr(),
                                    st), "dyprep")
    elif case in ("step-fp8", "step-fp16", "step-tf32"):
        # one full APA step (pre_step, forward, backward, ladder) through the
        # public API, between cudaProfilerStart/Stop after warm-up steps, for
        # `ncu --profile-from-start off` launch lists
        import torch.nn as nn
        from apa import APAConfig, APALinear, APAManager
        level = {"step-fp8": 0, "step-fp16": 1, "step-tf32": 2}[case]
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
        dy = torch.randn(M, N, device=dev, generator=g)
        if level == 1:
            dy = dy.half()
        cfg = APAConfig(device=str(dev), check_interval=1)
        torch.manual_seed(0)
        lin = APALinear(K, N, config=cfg)
        lin.level = level
        mgr = APAManager(nn.Sequential(lin), cfg)

        def step():
            mgr.pre_step()
            lin(x).backward(dy)
            x.grad = None
            mgr.post_backward_sync_and_eval()
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    elif case in ("step-gpt2m", "step-gpt-char"):
        # one eager GPT training step (pre_step, forward, backward, ladder,
        # AdamW) between cudaProfilerStart/Stop, after warm-up steps
        import torch.nn as nn
        import torch.nn.functional as F
        import apa
        from apa import APAManager
        cfgd = GPT_CONFIGS[case[len("step-"):]]
        model, cfg = build_gpt(torch, nn, F, apa, cfgd, dev)
        mgr = APAManager(model, cfg)
        opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=cfgd["lr"], weight_decay=0.01, fused=True)
        batches = gpt_batches(torch, cfgd, 0, dev)
        V = cfgd["vocab_pad"]

        def step(i):
            xb, yb = batches[i % len(batches)]
            mgr.pre_step()
            opt.zero_grad(set_to_none=True)
            loss = F.cross_entropy(model(xb).reshape(-1, V).float(), yb.reshape(-1))
            loss.backward()
            if mgr.post_backward_sync_and_eval():
                opt.step()
        for i in range(4):
            step(i)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        step(4)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    elif case == "step-vit":
        # one eager ViT training step between cudaProfilerStart/Stop, after warm-up steps
        import torch.nn as nn
        import torch.nn.functional as F
        import apa
        from apa import APAManager
        cfgd = VIT_CONFIG
        model, cfg = build_vit(torch, nn, F, apa, cfgd, dev)
        mgr = APAManager(model, cfg)
        opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=cfgd["lr"], weight_decay=0.01, fused=True)
        gi = torch.Generator().manual_seed(4321)
        B = cfgd["batch"]
        xb = torch.randn(B, cfgd["ch"], cfgd["img"], cfgd["img"], generator=gi).to(dev)
        yb = torch.randint(0, cfgd["classes"], (B,), generator=gi).to(dev)

        def step():
            mgr.pre_step()
            opt.zero_grad(set_to_none=True)
            F.cross_entropy(model(xb).float(), yb).backward()
            if mgr.post_backward_sync_and_eval():
                opt.step()
        for _ in range(4):
            step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    elif case == "adamw-fp8":
        # AdamW on the 4096x4096 master fused with its FP8 working copies
        p = torch.randn(N, K, device=dev, generator=g) * 0.02
        gr = torch.randn(N, K, device=dev, generator=g) * 1e-3
        m, v = torch.zeros_like(p), torch.zeros_like(p)
        wq = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=dev)
        wqt = torch.empty(K, N, dtype=torch.float8_e4m3fn, device=dev)
        amax = torch.zeros(1, device=dev)
        for i in range(3):
            _lib.check(lib.apa_adamw_cast(p.data_ptr(), gr.data_ptr(), m.data_ptr(), v.data_ptr(), N, K, K, 1e-3,
                                          0.9, 0.999, 1e-8, 0.01, i + 1, wq.data_ptr(), _lib.DT_E4M3, K,
                                          wqt.data_ptr(), N, amax.data_ptr(), st), "adamw_cast")
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    print(json.dumps({"profile_case": case, "ok": True}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gpt", default="gpt-char,gpt2m",
                    help="GPT training workloads also timed (tokens/s), comma-separated; '' for none")
    ap.add_argument("--gpt-steps", type=int, default=10)
    ap.add_argument("--no-vit", dest="vit", action="store_false",
                    help="skip the ViT classifier workload (images/s)")
    ap.add_argument("--gpt-eager", action="store_true", help="time the GPT workloads without CUDA-graph replay")
    ap.add_argument("--gpt-optimizer", choices=["auto", "torch", "apa"], default="auto",
                    help="optimizer of the GPT workloads: torch.optim.AdamW(fused), apa.optim.APAAdamW, or auto "
                         "(APAAdamW for GPT-2-medium, torch's for the char model)")
    ap.add_argument("--dp-bucket-bytes", type=int, default=64 << 20,
                    help="data parallel gradient bucket size in bytes")
    ap.add_argument("--dp-block-bytes", type=int, default=0,
                    help="data parallel: APALinear weights this large have their gradient computed and all-reduced "
                         "in row blocks (0, the default: one all-reduce per bucket after the whole gradient; "
                         "row blocks measured slower on 2 GPUs)")
    ap.add_argument("--dp-nvls", type=int, default=0,
                    help="data parallel: average large APALinear weight gradients through NVLink SHARP with the "
                         "library's own kernels (1, where the GPUs have NVLink multicast) or in NCCL buckets only "
                         "(0, the default; the two measured level on two GPUs)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch the library's kernels in plain stream order instead of with programmatic dependent "
                         "launch (each kernel's launch and prologue overlapping the end of the one before)")
    ap.add_argument("--eager", action="store_true",
                    help="time the APALinear steps without CUDA-graph replay (every launch from the host)")
    ap.add_argument("--profile-case", default=None,
                    help="run a few launches of one kernel for an ncu capture (gemm-fp8|gemm-fp16|gemm-tf32|gemm-fp8-k1024|"
                         "gemm-table: timing table of the GPT-2-medium FP8 GEMMs against cuBLASLt|"
                         "dgrad-fp8|dgrad-fp16|dgrad-tf32|wgrad-fp8|wgrad-fp16|wgrad-tf32|cast|dyprep|cast-tf32|"
                         "dyprep-tf32|adamw-fp8), "
                         "or one profiled step (step-fp8|step-fp16|step-tf32|step-gpt2m|step-gpt-char|step-vit)")
    args = ap.parse_args()
    if args.profile_case == "gemm-table":
        gemm_table()
        return
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.warmup < 3:
        args.warmup = 3
    args.gpt = [g for g in args.gpt.split(",") if g]
    # libraries (NCCL, the reference's event logger) print to stdout; route the
    # process's fd 1 to stderr while working so stdout carries one JSON line
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        out = run_reference(args) if args.impl == "reference" else run_ours(args)
    finally:
        sys.stdout.flush()
        os.dup2(json_fd, 1)
        os.close(json_fd)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
