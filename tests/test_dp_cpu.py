"""Data-parallel trainer logic on CPU gloo ranks (world_size 2).

The data-parallel equivalence check, scaled down: global batch sharded evenly, rank r
draws its shard from seed+r, MSE per shard, all-reduced gradients, SGD lr
1e-2; after 10 steps loss and weights match a single-process run over the
concatenated batch.  torch.nn.GRU stands in for the per-rank compute (the DP
logic is module-agnostic; the CUDA module is exercised by the GPU tests).
"""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rnn_kernel_b200.train import DataParallelTrainer, flatten_parameters_

I, H, T, GLOBAL_B, STEPS, LR, SEED = 5, 8, 6, 8, 10, 1e-2, 1234


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(rank, step, b):
    g = torch.Generator().manual_seed(SEED + rank + 1000 * step)
    return torch.randn(b, T, I, generator=g), torch.randn(b, T, H, generator=g)


def _worker(rank, world, port, out_path, layers=1, overlap=True):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0 if rank == 0 else 99)  # weights differ until the broadcast
    model = torch.nn.GRU(I, H, num_layers=layers, batch_first=True)
    tr = DataParallelTrainer(model, lr=LR, overlap=overlap)
    assert bool(tr._buckets) == (bool(overlap) and layers > 1)
    losses = []
    for step in range(STEPS):
        if overlap == "toggle":
            # what GraphedTrainStep does to the trainer, every other step: the
            # per-layer hooks stay registered but the whole buffer is reduced
            # after the backward (used to raise IndexError from the hooks)
            tr.overlap_active = step % 2 == 1
        x, y = _shard(rank, step, GLOBAL_B // world)
        loss = tr.step(x, y)
        t = loss.clone()
        dist.all_reduce(t)
        losses.append(float(t) / world)
    if rank == 0:
        torch.save({"flat": tr.flat.clone(), "losses": losses}, out_path)
    dist.destroy_process_group()


def _single(world, layers=1):
    torch.manual_seed(0)
    model = torch.nn.GRU(I, H, num_layers=layers, batch_first=True)
    tr = DataParallelTrainer(model, lr=LR)
    losses = []
    for step in range(STEPS):
        xs, ys = zip(*[_shard(r, step, GLOBAL_B // world) for r in range(world)])
        losses.append(float(tr.step(torch.cat(xs), torch.cat(ys))))
    return tr.flat, losses


def test_flatten_parameters_views():
    m = torch.nn.GRU(3, 4, num_layers=2, batch_first=True)
    before = [p.detach().clone() for p in m.parameters()]
    flat, grad = flatten_parameters_(m)
    assert flat.numel() == sum(p.numel() for p in before)
    for p, b in zip(m.parameters(), before):
        assert torch.equal(p, b)
        assert p.data_ptr() >= flat.data_ptr() and p.grad.data_ptr() >= grad.data_ptr()
    out, _ = m(torch.randn(2, 3, 3))
    out.sum().backward()
    assert grad.abs().sum() > 0  # autograd accumulated into the flat buffer in place


@pytest.mark.timeout(300)
@pytest.mark.parametrize("layers,overlap", [(1, True), (2, True), (2, False), (2, "toggle")])
def test_dp_gloo_two_ranks_matches_single_process(layers, overlap):
    # layers=2, overlap=True: per-layer buckets all-reduced asynchronously
    # from post-accumulate-grad hooks while the lower layer's backward runs.
    world = 2
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "r0.pt")
        mp.spawn(_worker, args=(world, _free_port(), path, layers, overlap), nprocs=world, join=True)
        res = torch.load(path)
    flat1, losses1 = _single(world, layers)
    torch.testing.assert_close(res["flat"], flat1, rtol=1e-5, atol=1e-6)
    for a, b in zip(res["losses"], losses1):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(b))


def _failing_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    model = torch.nn.GRU(I, H, batch_first=True)
    tr = DataParallelTrainer(model, lr=LR)
    if rank == 1:
        raise RuntimeError("rank 1 fails between steps")
    x, y = _shard(rank, 0, 2)
    tr.step(x, y)  # rank 0's all-reduce must error out (peer gone), not hang


@pytest.mark.timeout(300)
def test_dp_rank_failure_surfaces_as_error():
    with pytest.raises(Exception):
        mp.spawn(_failing_worker, args=(2, _free_port()), nprocs=2, join=True)
