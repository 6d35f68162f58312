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


@pytest.mark.parametrize("layers,include_update", [(1, False), (2, False), (1, True), (2, True)])
def test_graphed_steps_match_eager_steps(layers, include_update):
    from rnn_kernel_b200 import GraphedTrainStep

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(3)
    host = [(torch.randn(5, 11, 24, generator=g), torch.randn(5, 11, 40, generator=g)) for _ in range(6)]

    def make():
        torch.manual_seed(21)
        return DataParallelTrainer(GRU(24, 40, num_layers=layers).to(dev), lr=1e-2)

    # eager reference: 3 warm-up steps on batch 0 (what the capture warm-up
    # does), then one step per batch
    ref = make()
    x0, y0 = (t.to(dev) for t in host[0])
    for _ in range(3):
        ref.step(x0, y0)
    ref_losses = [float(ref.step(x.to(dev), y.to(dev))) for x, y in host]

    tr = make()
    xs, ys = x0.clone(), y0.clone()
    gs = GraphedTrainStep(tr, [(xs, ys)], warmup=3, include_update=include_update)
    losses = []
    for x, y in host:
        xs.copy_(x)
        ys.copy_(y)
        losses.append(float(gs.step(0)))
    assert losses == ref_losses
    assert torch.equal(tr.flat, ref.flat)


def test_graphed_steps_on_prefetcher_buffers():
    from rnn_kernel_b200 import GraphedTrainStep

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(4)
    host = [(torch.randn(3, 7, 16, generator=g).pin_memory(), torch.randn(3, 7, 32, generator=g).pin_memory())
            for _ in range(5)]
    torch.manual_seed(5)
    ref = DataParallelTrainer(GRU(16, 32).to(dev), lr=1e-2)
    torch.manual_seed(5)
    tr = DataParallelTrainer(GRU(16, 32).to(dev), lr=1e-2)

    pf = HostBatchPrefetcher(dev)
    for _ in range(2):  # allocate both buffer sets with batch 0
        pf.put(*host[0])
        pf.get()
    torch.cuda.synchronize()
    gs = GraphedTrainStep(tr, [pf._bufs[0], pf._bufs[1]], warmup=1)
    x0, y0 = (t.to(dev) for t in host[0])
    for _ in range(2):  # the capture warm-up: one step per buffer set, batch 0
        ref.step(x0, y0)
    pf.put(*host[0])
    losses, ref_losses = [], []
    for k in range(len(host)):
        pf.get()
        slot = pf._in_use
        if k + 1 < len(host):
            pf.put(*host[k + 1])
        losses.append(float(gs.step(slot)))
        ref_losses.append(float(ref.step(host[k][0].to(dev), host[k][1].to(dev))))
    assert losses == ref_losses
    assert torch.equal(tr.flat, ref.flat)
