"""The library's one-pass MSE loss against torch's F.mse_loss (the training
harness's loss, rnn_benchmark.py:636): value, gradient, odd sizes, unaligned
storage, a non-unit upstream gradient, and graph capture."""
import pytest
import torch
import torch.nn.functional as F

from rnn_kernel_b200 import mse_loss

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(64, 512, 256), (3, 7, 5), (1, 1, 1), (2, 9, 130)])
@pytest.mark.parametrize("offset", [0, 1])
def test_mse_matches_torch(shape, offset):
    torch.manual_seed(sum(shape) + offset)
    n = 1
    for s in shape:
        n *= s
    base = torch.randn(n + offset, device="cuda")
    out = base[offset:].view(shape).clone().requires_grad_(True) if offset == 0 else base[offset:].view(shape)
    out = out.detach().requires_grad_(True)
    y = torch.randn(shape, device="cuda")
    ref_out = out.detach().clone().requires_grad_(True)
    loss = mse_loss(out, y)
    ref = F.mse_loss(ref_out, y)
    # FP64 sum here, FP32 tree in torch: equal to FP32 rounding of a long sum
    torch.testing.assert_close(loss, ref, rtol=2e-6, atol=0)
    exact = F.mse_loss(out.detach().double(), y.double()).float()
    torch.testing.assert_close(loss, exact, rtol=2e-7, atol=0)
    (3.0 * loss).backward()
    (3.0 * ref).backward()
    torch.testing.assert_close(out.grad, ref_out.grad, rtol=1e-6, atol=1e-12)


def test_mse_in_graph_capture():
    torch.manual_seed(0)
    out = torch.randn(8, 16, 32, device="cuda", requires_grad=True)
    y = torch.randn(8, 16, 32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mse_loss(out, y).backward()
    torch.cuda.current_stream().wait_stream(s)
    out.grad = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        loss = mse_loss(out, y)
        loss.backward()
    out.grad.zero_()
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(loss, F.mse_loss(out.detach(), y), rtol=2e-6, atol=0)
    torch.testing.assert_close(out.grad, 2.0 * (out.detach() - y) / out.numel(), rtol=1e-6, atol=1e-12)


def test_mse_rejects():
    with pytest.raises(ValueError):
        mse_loss(torch.zeros(2, 3, device="cuda"), torch.zeros(3, 2, device="cuda"))
    with pytest.raises(RuntimeError):
        mse_loss(torch.zeros(2, 3, device="cuda", dtype=torch.float64), torch.zeros(2, 3, device="cuda",
                                                                                 dtype=torch.float64))
