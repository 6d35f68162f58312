"""MSE loss of the GRU output on the CUDA library (one pass forward, one pass
backward), the loss of the reference's training harness (``F.mse_loss(pred,
y)``: rnn_benchmark.py:636, :657, :680; tests/test_sequence_chunking.py:27-28).

``mse_loss(out, target)`` equals ``F.mse_loss(out, target)`` (mean reduction)
up to the summation order of the loss value (here FP64, deterministic); the
gradient is computed as torch does, ``(2 / n) * (out - target) * g``.  FP32
CUDA tensors only, ``target`` without gradient; the library must be present.
"""
from __future__ import annotations

import torch

from . import _lib


class MSELossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        if out.shape != target.shape:
            raise ValueError("out and target must have the same shape.")
        if out.dtype != torch.float32 or target.dtype != torch.float32 or not out.is_cuda or not target.is_cuda:
            raise RuntimeError("mse_loss: FP32 CUDA tensors are required.")
        o = out.contiguous()
        t = target.contiguous()
        n = o.numel()
        lib = _lib.load()
        ws = torch.empty(max(1, lib.gru_mse_workspace_bytes(n)), dtype=torch.uint8, device=o.device)
        loss = torch.empty((), dtype=torch.float32, device=o.device)
        stream = torch.cuda.current_stream(o.device).cuda_stream
        _lib.check(lib.gru_mse_loss(o.data_ptr(), t.data_ptr(), n, loss.data_ptr(), ws.data_ptr(), ws.numel(),
                                    stream), "gru_mse_loss")
        ctx.save_for_backward(o, t)
        return loss

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        o, t = ctx.saved_tensors
        g = g.detach().to(torch.float32).contiguous()
        dout = torch.empty_like(o)
        stream = torch.cuda.current_stream(o.device).cuda_stream
        _lib.check(_lib.load().gru_mse_loss_backward(o.data_ptr(), t.data_ptr(), g.data_ptr(), dout.data_ptr(),
                                                     o.numel(), stream), "gru_mse_loss_backward")
        return dout, None


def mse_loss(out: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Mean squared error on the CUDA library (see the module docstring)."""
    if target.requires_grad:
        raise ValueError("mse_loss: target must not require grad.")
    return MSELossFunction.apply(out, target)
