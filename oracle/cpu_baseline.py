"""CPU baseline timing (test / benchmark infrastructure, never the product).

The reference's own CPU path for this workload is stock ``torch.nn.GRU``
driven by its harness (``rnn_benchmark.py --device cpu``: model built at
``rnn_benchmark.py:198-207``, ``train_step`` at ``:628-639``, tokens/s =
B*T*steps/s at ``:754``).  This module times exactly that on the host cores
with the benchmark's loss/optimizer (MSE against an N(0,1) target, SGD lr 1e-2),
all threads, ``time.perf_counter`` around each step.
"""
from __future__ import annotations

import os
import platform
import time


def cpu_model_name() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def time_cpu_train_step(B: int, T: int, I: int, H: int, warmup: int = 1, steps: int = 2,
                        threads: int | None = None, seed: int = 0) -> dict:
    import torch
    import torch.nn.functional as F

    threads = threads or os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        torch.manual_seed(seed)
        model = torch.nn.GRU(I, H, batch_first=True)
        opt = torch.optim.SGD(model.parameters(), lr=1e-2)
        x = torch.randn(B, T, I)
        y = torch.randn(B, T, H)

        def step():
            opt.zero_grad(set_to_none=True)
            out, _ = model(x)
            loss = F.mse_loss(out, y)
            loss.backward()
            opt.step()
            return float(loss)

        for _ in range(warmup):
            step()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            step()
            times.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(prev)
    s = sum(times) / len(times)
    return {
        "value": B * T / s,
        "ms_per_step": 1e3 * s,
        "cores": threads,
        "cpu_model": cpu_model_name(),
        "steps": steps,
        "warmup": warmup,
    }
