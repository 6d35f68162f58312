"""Data-parallel training on 2 GPUs with NCCL (scaled down): the global batch is sharded evenly, rank r draws its shard from
seed + r, each rank runs the B200 GRU on its own GPU, gradients are
all-reduced, SGD lr 1e-2; after 10 steps the loss and the weights match a
single-process run over the concatenated batch.  Skipped with fewer than 2
GPUs."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

I, H, T, GLOBAL_B, STEPS, LR, SEED, WARM = 32, 64, 24, 16, 10, 1e-2, 77, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(rank, step, b, dev):
    g = torch.Generator().manual_seed(SEED + rank + 1000 * step)
    return torch.randn(b, T, I, generator=g).to(dev), torch.randn(b, T, H, generator=g).to(dev)


def _worker(rank, world, port, out_path, layers=1, graphed=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from rnn_kernel_b200 import GRU, DataParallelTrainer, GraphedTrainStep

    torch.manual_seed(0)
    model = GRU(I, H, num_layers=layers).cuda()
    tr = DataParallelTrainer(model, lr=LR)
    assert bool(tr._buckets) == (layers > 1)  # per-layer overlapped all-reduce
    losses = []
    gs = None
    if graphed:
        # replayed steps (hooks off, one all-reduce after the replay); the
        # capture warm-up trains on step 0's shard, so the reference starts
        # with the same number of extra steps on it
        xs, ys = _shard(rank, 0, GLOBAL_B // world, "cuda")
        gs = GraphedTrainStep(tr, [(xs, ys)], warmup=WARM, capture_error_mode="thread_local")
    for step in range(STEPS):
        x, y = _shard(rank, step, GLOBAL_B // world, "cuda")
        if gs is not None:
            xs.copy_(x)
            ys.copy_(y)
            loss = gs.step(0).clone()
        else:
            loss = tr.step(x, y)
        dist.all_reduce(loss)
        losses.append(float(loss) / world)
    if rank == 0:
        torch.save({"flat": tr.flat.cpu(), "losses": losses}, out_path)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("layers,graphed", [(1, False), (2, False), (2, "replay")])
def test_dp_two_gpus_matches_single_gpu(layers, graphed):
    from rnn_kernel_b200 import GRU, DataParallelTrainer

    world = 2
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "r0.pt")
        mp.spawn(_worker, args=(world, _free_port(), path, layers, graphed), nprocs=world, join=True)
        res = torch.load(path)
    torch.manual_seed(0)
    model = GRU(I, H, num_layers=layers).cuda()
    tr = DataParallelTrainer(model, lr=LR)
    if graphed:
        xs, ys = zip(*[_shard(r, 0, GLOBAL_B // world, "cuda") for r in range(world)])
        for _ in range(WARM):
            tr.step(torch.cat(xs), torch.cat(ys))
    losses = []
    for step in range(STEPS):
        xs, ys = zip(*[_shard(r, step, GLOBAL_B // world, "cuda") for r in range(world)])
        losses.append(float(tr.step(torch.cat(xs), torch.cat(ys))))
    torch.testing.assert_close(res["flat"], tr.flat.cpu(), rtol=1e-4, atol=1e-5)
    for a, b in zip(res["losses"], losses):
        assert abs(a - b) <= 1e-4 * abs(b) + 1e-6


def _bucket_worker(rank, world, port, out_path):
    # one rank: the per-layer bucket hooks and their NCCL all-reduces run on a
    # single GPU; the SUM over one rank leaves the gradients unchanged, so the
    # step must equal the plain one exactly
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    from rnn_kernel_b200 import GRU, DataParallelTrainer

    def run(bucketed):
        torch.manual_seed(0)
        tr = DataParallelTrainer(GRU(I, H, num_layers=3).cuda(), lr=LR)
        if bucketed:
            tr._install_bucket_hooks()
            assert len(tr._buckets) == 3 and tr.overlap_active
        losses, started = [], []
        for step in range(4):
            x, y = _shard(0, step, 6, "cuda")
            loss = tr.forward_backward(x, y)
            started.append(len(tr._works))  # all-reduces the hooks launched during the backward
            tr.reduce_and_update()
            losses.append(float(loss))
        return tr.flat.cpu(), losses, started

    a = run(True)
    b = run(False)
    torch.save({"a": a, "b": b}, out_path)
    dist.destroy_process_group()


def test_per_layer_bucket_hooks_one_gpu():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "r.pt")
        mp.spawn(_bucket_worker, args=(1, _free_port(), path), nprocs=1, join=True)
        res = torch.load(path)
    (wa, la, started), (wb, lb, none) = res["a"], res["b"]
    # every layer's bucket was all-reduced from its hook during the backward
    assert started == [3, 3, 3, 3] and none == [0, 0, 0, 0]
    assert la == lb
    assert torch.equal(wa, wb)
