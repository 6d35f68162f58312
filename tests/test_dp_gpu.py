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

I, H, T, GLOBAL_B, STEPS, LR, SEED = 32, 64, 24, 16, 10, 1e-2, 77


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(rank, step, b, dev):
    g = torch.Generator().manual_seed(SEED + rank + 1000 * step)
    return torch.randn(b, T, I, generator=g).to(dev), torch.randn(b, T, H, generator=g).to(dev)


def _worker(rank, world, port, out_path, layers=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from rnn_kernel_b200 import GRU, DataParallelTrainer

    torch.manual_seed(0)
    model = GRU(I, H, num_layers=layers).cuda()
    tr = DataParallelTrainer(model, lr=LR)
    assert bool(tr._buckets) == (layers > 1)  # per-layer overlapped all-reduce
    losses = []
    for step in range(STEPS):
        x, y = _shard(rank, step, GLOBAL_B // world, "cuda")
        loss = tr.step(x, y)
        dist.all_reduce(loss)
        losses.append(float(loss) / world)
    if rank == 0:
        torch.save({"flat": tr.flat.cpu(), "losses": losses}, out_path)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("layers", [1, 2])
def test_dp_two_gpus_matches_single_gpu(layers):
    from rnn_kernel_b200 import GRU, DataParallelTrainer

    world = 2
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "r0.pt")
        mp.spawn(_worker, args=(world, _free_port(), path, layers), nprocs=world, join=True)
        res = torch.load(path)
    torch.manual_seed(0)
    model = GRU(I, H, num_layers=layers).cuda()
    tr = DataParallelTrainer(model, lr=LR)
    losses = []
    for step in range(STEPS):
        xs, ys = zip(*[_shard(r, step, GLOBAL_B // world, "cuda") for r in range(world)])
        losses.append(float(tr.step(torch.cat(xs), torch.cat(ys))))
    torch.testing.assert_close(res["flat"], tr.flat.cpu(), rtol=1e-4, atol=1e-5)
    for a, b in zip(res["losses"], losses):
        assert abs(a - b) <= 1e-4 * abs(b) + 1e-6
