"""HostBatchPrefetcher: order and contents of the staged batches, and training
through it matches training on device-resident inputs exactly."""
import pytest
import torch

from rnn_kernel_b200 import GRU, DataParallelTrainer, HostBatchPrefetcher

pytestmark = pytest.mark.gpu


def test_batches_arrive_in_order():
    dev = torch.device("cuda", 0)
    host = [(torch.full((4, 3, 5), float(i)).pin_memory(), torch.full((7,), -float(i)).pin_memory())
            for i in range(5)]
    pf = HostBatchPrefetcher(dev)
    pf.put(*host[0])
    seen = []
    for k in range(5):
        xd, yd = pf.get()
        if k + 1 < 5:
            pf.put(*host[k + 1])
        # work on the compute stream that reads the buffers, then a copy back
        seen.append(((xd * 2).cpu(), (yd + 1).cpu()))
    for k, (a, b) in enumerate(seen):
        torch.testing.assert_close(a, torch.full((4, 3, 5), 2.0 * k))
        torch.testing.assert_close(b, torch.full((7,), 1.0 - k))


def test_get_without_put_and_overfill_raise():
    pf = HostBatchPrefetcher(torch.device("cuda", 0))
    with pytest.raises(RuntimeError):
        pf.get()
    t = torch.zeros(3).pin_memory()
    pf.put(t)
    pf.put(t)
    with pytest.raises(RuntimeError):
        pf.put(t)
    assert pf.get().shape == (3,)


def test_training_through_prefetcher_matches_device_inputs():
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(7)
    batches = [(torch.randn(6, 9, 16, generator=g), torch.randn(6, 9, 32, generator=g)) for _ in range(4)]

    def run(use_prefetcher):
        torch.manual_seed(11)
        model = GRU(16, 32).to(dev)
        tr = DataParallelTrainer(model, lr=1e-2)
        losses = []
        if use_prefetcher:
            pinned = [(x.pin_memory(), y.pin_memory()) for x, y in batches]
            pf = HostBatchPrefetcher(dev)
            pf.put(*pinned[0])
            for k in range(len(batches)):
                xd, yd = pf.get()
                if k + 1 < len(batches):
                    pf.put(*pinned[k + 1])
                losses.append(float(tr.step(xd, yd)))
        else:
            for x, y in batches:
                losses.append(float(tr.step(x.to(dev), y.to(dev))))
        return losses, tr.flat.detach().cpu()

    l1, w1 = run(True)
    l2, w2 = run(False)
    assert l1 == l2
    assert torch.equal(w1, w2)
