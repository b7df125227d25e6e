"""APAAdamW: AdamW fused with the next step's working-copy cast.

* apa_adamw_cast against torch.optim.AdamW on the same tensors: p, m, v agree
  to fp32 rounding over several steps; the working copy, its transpose and
  the weight amax equal, bit for bit, what the library's own cast makes of
  the updated master.
* Training with APAAdamW against torch.optim.AdamW: the same decisions and
  weights to fp32 rounding, with every APALinear weight updated by the fused
  kernel and pre_step skipping those weights' casts."""
import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

WORK = {0: (torch.float8_e4m3fn, 3), 1: (torch.float16, 1), 2: (torch.float32, 4)}


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def bits(t):
    return t.view(torch.uint8 if t.element_size() == 1 else (torch.int16 if t.element_size() == 2 else torch.int32))


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("copies", ["both", "row", "transposed"])
@pytest.mark.parametrize("shape", [(128, 64), (200, 136), (33, 20), (1024, 512), (4096, 1024)])
def test_adamw_cast_kernel(L, rung, copies, shape):
    N, K = shape
    g0 = torch.Generator(device="cuda").manual_seed(N * 7 + rung)
    p = (torch.randn(N, K, device="cuda", generator=g0) * 0.05).contiguous()
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, foreach=False)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    wdt, code = WORK[rung]
    es = torch.empty((), dtype=wdt).element_size()

    def alloc(rows, cols):        # 16-byte row pitch, as APALinear allocates its working copies
        ld = (cols * es + 15) // 16 * 16 // es
        return torch.empty(rows, ld, dtype=wdt, device="cuda")[:, :cols]

    if copies != "both" and shape not in ((200, 136), (1024, 512)):
        pytest.skip("one copy: two shapes suffice")
    wq, wqt = alloc(N, K), alloc(K, N)
    want_q, want_t = copies != "transposed", copies != "row"
    amax = torch.zeros(1, device="cuda")
    s = L.stream_handle()
    for step in range(1, 4):
        g = torch.randn(N, K, device="cuda", generator=g0) * 0.01
        ref.grad = g.clone()
        opt.step()
        amax.zero_()
        L.check(L.lib().apa_adamw_cast(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), N, K, K, 3e-3, 0.9,
                                       0.95, 1e-8, 0.1, step, wq.data_ptr() if want_q else None, code, wq.stride(0),
                                       wqt.data_ptr() if want_t else None, wqt.stride(0), amax.data_ptr(), s),
                "apa_adamw_cast")
        torch.cuda.synchronize()
        st = opt.state[ref]
        for got, want in ((p, ref.detach()), (m, st["exp_avg"]), (v, st["exp_avg_sq"])):
            err = ((got - want).abs().max() / want.abs().max().clamp_min(1e-30)).item()
            assert err < 2e-6, (step, err)
        # the working copies are the library's cast of the updated master
        cq, cqt = alloc(N, K), alloc(K, N)
        camax = torch.zeros(1, device="cuda")
        L.check(L.lib().apa_cast(p.data_ptr(), L.DT_F32, N, K, K, cq.data_ptr(), code, cq.stride(0), cqt.data_ptr(),
                                 cqt.stride(0), camax.data_ptr(), None, 0, None, None, s), "apa_cast")
        torch.cuda.synchronize()
        if want_q:
            assert torch.equal(bits(wq.contiguous()), bits(cq.contiguous()))
        if want_t:
            assert torch.equal(bits(wqt.contiguous()), bits(cqt.contiguous()))
        assert amax.item() == camax.item()
    assert L.device_status() == 0


class LayerNorm32(nn.LayerNorm):
    def forward(self, x):
        return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps)


def _train(use_apa_opt, steps=10, spike=6):
    from apa import APAConfig, APALinear, APAManager
    from apa.optim import APAAdamW
    cfg = APAConfig(device="cuda", check_interval=2)
    torch.manual_seed(0)
    model = nn.Sequential(APALinear(64, 128, config=cfg), nn.ReLU(), LayerNorm32(128),
                          APALinear(128, 32, config=cfg)).cuda()
    mgr = APAManager(model, cfg)
    params = mgr.get_trainable_parameters()
    opt = APAAdamW(mgr, lr=2e-3, weight_decay=0.05) if use_apa_opt else \
        torch.optim.AdamW(params, lr=2e-3, weight_decay=0.05)
    g = torch.Generator().manual_seed(3)
    keeps, levels = [], []
    for i in range(steps):
        x = torch.randn(96, 64, generator=g)
        if i == spike:
            x[0, :8] *= 1e4                        # an overflow: skip + escalation
        y = torch.randint(0, 32, (96,), generator=g)
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(model(x.cuda()).float(), y.cuda()).backward()
        keep = mgr.post_backward_sync_and_eval()
        if keep:
            opt.step()
        keeps.append(keep)
        levels.append([m.level for m in mgr.apa_modules.values()])
    torch.cuda.synchronize()
    return keeps, levels, [p.detach().clone() for p in params], opt


def test_training_matches_torch_adamw():
    k1, l1, p1, opt = _train(True)
    k2, l2, p2, _ = _train(False)
    assert k1 == k2 and l1 == l2
    assert not k1[6] and l1[6] != l1[5]            # the spike was skipped and escalated a layer
    for a, b in zip(p1, p2):
        assert ((a - b).abs().max() / b.abs().max()).item() < 1e-4
    # both weights fused on every kept step except right after the escalation
    # (the layer's buffers follow the new level only from the next pre_step)
    assert opt.fused_steps >= 2 * (sum(k1) - 1)
