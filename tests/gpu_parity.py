"""Shared parity harness for the GPU tests: run torch.nn.GRU FP32 on the CPU
(the reference's parity anchor, tests/test_a100_prod.py:84-126) and the B200
module on cuda:0 on the same seeded inputs, and compare every output and
gradient within the north-star tolerance rtol 1e-4 / atol 1e-5."""
from __future__ import annotations

import torch

from rnn_kernel_b200 import from_torch_gru

RTOL, ATOL = 1e-4, 1e-5


def run_pair(I, H, L, B, T, seed, loss="random", h0_scale=1.0, ref_dtype=torch.float32):
    torch.manual_seed(seed)
    ref = torch.nn.GRU(I, H, num_layers=L, batch_first=True)
    x = torch.randn(B, T, I)
    h0 = h0_scale * torch.randn(L, B, H) if h0_scale else torch.zeros(L, B, H)
    go = torch.randn(B, T, H)
    gh = torch.randn(L, B, H)
    tgt = torch.randn(B, T, H)

    def run(model, dev, dtype):
        xx = x.to(dev, dtype).requires_grad_(True)
        hh = h0.to(dev, dtype).requires_grad_(True)
        out, hn = model(xx, hh)
        if loss == "random":
            torch.autograd.backward([out, hn], [go.to(dev, dtype), gh.to(dev, dtype)])
        elif loss == "mse":
            torch.nn.functional.mse_loss(out, tgt.to(dev, dtype)).backward()
        elif loss == "sumsq":
            (out * out).sum().backward()
        elif loss == "hn_only":
            hn.backward(gh.to(dev, dtype))
        else:
            raise ValueError(loss)
        res = {"out": out, "hn": hn, "dx": xx.grad, "dh0": hh.grad}
        for n, p in model.named_parameters():
            res["d" + n] = p.grad
        return {k: v.detach().double().cpu() for k, v in res.items()}

    ours = from_torch_gru(ref.cuda())
    mine = run(ours, "cuda", torch.float32)
    ref_cpu = ref.cpu().to(ref_dtype)
    theirs = run(ref_cpu, "cpu", ref_dtype)
    return mine, theirs


def assert_parity(mine, theirs, rtol=RTOL, atol=ATOL):
    bad = []
    for k in theirs:
        a, b = mine[k], theirs[k]
        assert a.shape == b.shape, (k, a.shape, b.shape)
        if not torch.allclose(a, b, rtol=rtol, atol=atol):
            err = (a - b).abs()
            lim = atol + rtol * b.abs()
            bad.append(f"{k}: max|d|={err.max():.3e} worst ratio={(err / lim).max():.2f} max|ref|={b.abs().max():.3e}")
    assert not bad, "\n".join(bad)
