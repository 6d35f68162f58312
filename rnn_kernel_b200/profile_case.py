"""Run a small GRU train step case on cuda:0, for profilers.

    python -m rnn_kernel_b200.profile_case --batch 64 --seq 128

Two iterations of forward + MSE + backward of a 1-layer I=H=256 GRU (sizes
configurable), synchronised at the end.  Meant to be wrapped by ncu / nsys:
it keeps the device footprint small (a few hundred MB) so a full-metric
capture of its kernels ends quickly.
"""
from __future__ import annotations

import argparse

import torch

from . import GRU


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--input", type=int, default=256)
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--iters", type=int, default=2)
    a = ap.parse_args()
    torch.manual_seed(0)
    m = GRU(a.input, a.hidden).cuda()
    x = torch.randn(a.batch, a.seq, a.input, device="cuda")
    y = torch.randn(a.batch, a.seq, a.hidden, device="cuda")
    for _ in range(a.iters):
        out, _ = m(x)
        torch.nn.functional.mse_loss(out, y).backward()
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
