"""The reference benchmark harness's own uses of the GRU, on the CUDA path,
checked against torch float64 (the truth) at rtol 1e-4 / atol 1e-5:

* carried-state chunked sequences (``sequence_chunk_len``): the sequence is
  fed chunk by chunk with the hidden state of the previous chunk carried in,
  and the loss and every gradient must equal one full-sequence pass through
  torch's float64 ``nn.GRU`` (ref tests/test_sequence_chunking.py:17-35,
  rnn_benchmark.py:512-520);
* the quick-check training loop: GRU + ``Linear(H, 1)`` head, MSE against a
  target y[B, T], AdamW(lr 3e-4, weight decay 1e-4), two steps (ref
  rnn_benchmark.py:510, :525, :628-639, :722, :997).
"""
import copy

import pytest
import torch
import torch.nn.functional as F

from rnn_kernel_b200 import from_torch_gru

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5


class _Model(torch.nn.Module):
    """GRU + Linear(H, 1) head, optionally fed in chunks with carried state."""

    def __init__(self, rnn, hidden, chunk):
        super().__init__()
        self.rnn, self.chunk = rnn, chunk
        self.head = torch.nn.Linear(hidden, 1)

    def forward(self, x):
        if self.chunk and x.size(1) > self.chunk:
            outs, h = [], None
            for s in range(0, x.size(1), self.chunk):
                o, h = self.rnn(x[:, s:s + self.chunk], h)
                outs.append(o)
            out = torch.cat(outs, 1)
        else:
            out, _ = self.rnn(x)
        return self.head(out).squeeze(-1)


def _pair(I, H, L, chunk, seed):
    torch.manual_seed(seed)
    gru = torch.nn.GRU(I, H, num_layers=L, batch_first=True)
    truth = _Model(copy.deepcopy(gru), H, 0).double()
    ours = _Model(from_torch_gru(copy.deepcopy(gru).cuda()), H, chunk).cuda()
    ours.head.load_state_dict(truth.head.state_dict())
    return ours, truth


def _close(name, a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    err = (a - b).abs()
    lim = ATOL + RTOL * b.abs()
    assert bool((err <= lim).all()), f"{name}: max|d|={float(err.max()):.3e} worst ratio={float((err / lim).max()):.2f}"


@pytest.mark.parametrize("I,H,L,B,T,chunk", [(3, 5, 2, 2, 11, 4), (3, 40, 2, 2, 11, 4), (16, 130, 2, 8, 37, 8),
                                             (256, 256, 1, 16, 64, 16)])
def test_chunked_sequence_matches_full_bptt_fp64(I, H, L, B, T, chunk):
    ours, truth = _pair(I, H, L, chunk, seed=123 + H)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, T, I, generator=g)
    y = torch.randn(B, T, generator=g)
    xo = x.cuda().requires_grad_(True)
    xt = x.double().requires_grad_(True)
    lo = F.mse_loss(ours(xo), y.cuda())
    lt = F.mse_loss(truth(xt), y.double())
    lo.backward()
    lt.backward()
    _close("loss", lo, lt)
    _close("dx", xo.grad, xt.grad)
    for (n, p), (_, q) in zip(ours.named_parameters(), truth.named_parameters()):
        _close("d" + n, p.grad, q.grad)


def test_quick_check_harness_head_adamw_two_steps():
    # quick-check shape: I = H = 16, B = 2, T = 8, seed 0, torch's default init
    I, H, B, T = 16, 16, 2, 8
    ours, truth = _pair(I, H, 1, 0, seed=0)
    g = torch.Generator().manual_seed(0)
    batches = [(torch.randn(B, T, I, generator=g), torch.randn(B, T, generator=g)) for _ in range(2)]
    opt_o = torch.optim.AdamW(ours.parameters(), lr=3e-4, weight_decay=1e-4)
    opt_t = torch.optim.AdamW(truth.parameters(), lr=3e-4, weight_decay=1e-4)
    for x, y in batches:
        for m, opt, dev, dt in ((ours, opt_o, "cuda", torch.float32), (truth, opt_t, "cpu", torch.float64)):
            opt.zero_grad(set_to_none=True)
            loss = F.mse_loss(m(x.to(dev, dt)), y.to(dev, dt))
            loss.backward()
            opt.step()
            if m is ours:
                lo = loss.detach()
            else:
                lt = loss.detach()
        _close("loss", lo, lt)
    for (n, p), (_, q) in zip(ours.named_parameters(), truth.named_parameters()):
        _close(n, p, q)
