"""Data-parallel GRU training over one process per GPU (NCCL over NVLink).

The reference has no distributed code; this is the B200 build's DP layer:
the global batch is sharded evenly across 1/2/4/8 GPUs, each rank takes the
MSE of its shard, gradients are all-reduced and SGD updates every replica.

Design: all parameters of the model are re-pointed into ONE flat FP32 buffer
and their ``.grad`` into ONE flat gradient buffer.  Autograd accumulates each
layer's gradients into that buffer in place, so a step is::

    grad.zero_(); loss = mse(model(x), y); loss.backward()
    all_reduce(grad, SUM)                      # one NCCL call, ~1.6 MB/layer
    flat_params.add_(grad, alpha=-lr / world)  # SGD on the mean gradient

i.e. one collective and one fused update kernel per step, independent of the
number of layers.  With ``overlap=True`` (default) and several layers, the
gradient buffer is reduced per layer instead: each layer's slice is
all-reduced asynchronously as soon as autograd has accumulated all of its
gradients (a post-accumulate-grad hook per parameter), so the upper layers'
reductions run while the lower layers' backward still computes; the update
waits for all of them.  The module is any ``nn.Module`` (the B200 :class:`GRU` on
GPUs; ``torch.nn.GRU`` on CPU ``gloo`` ranks in the tests of this logic).
"""
from __future__ import annotations

import re
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .loss import mse_loss


def flatten_parameters_(module: nn.Module):
    """Re-point every parameter of ``module`` into one flat buffer and give each
    a ``.grad`` view into one flat gradient buffer.  Returns ``(flat, grad)``."""
    params = [p for p in module.parameters() if p.requires_grad]
    if not params:
        raise ValueError("module has no trainable parameters")
    dev, dt = params[0].device, params[0].dtype
    flat = torch.empty(sum(p.numel() for p in params), device=dev, dtype=dt)
    grad = torch.zeros_like(flat)
    off = 0
    with torch.no_grad():
        for p in params:
            n = p.numel()
            flat[off:off + n].copy_(p.detach().reshape(-1))
            p.data = flat[off:off + n].view_as(p)
            p.grad = grad[off:off + n].view_as(p)
            off += n
    return flat, grad


class DataParallelTrainer:
    """SGD data-parallel trainer: shard-local fwd/bwd, one all-reduce, one update."""

    def __init__(self, module: nn.Module, lr: float = 1e-2,
                 process_group: Optional[dist.ProcessGroup] = None, overlap: bool = True) -> None:
        self.module = module
        self.lr = float(lr)
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_available() and dist.is_initialized() else 1
        self.flat, self.grad = flatten_parameters_(module)
        self._buckets: list = []   # [lo, hi) slices of the gradient buffer, one per layer
        self._pending: list = []   # parameters of each bucket not yet accumulated this step
        self._works: list = []
        self._in_step = False
        # Per-layer overlapped all-reduce; switched off (hooks stay registered
        # but return at once) by GraphedTrainStep, whose replay is followed by
        # one all-reduce of the whole buffer.
        self.overlap_active = False
        if self.world > 1:
            # Every rank starts from rank 0's weights.
            dist.broadcast(self.flat, src=0, group=process_group)
            if overlap:
                self._install_bucket_hooks()

    def _install_bucket_hooks(self) -> None:
        # Group the parameters by the layer suffix of their names (``_l{k}``,
        # nn.GRU convention); a layer's parameters must be contiguous in the
        # flat buffer.  One bucket only: nothing to overlap, keep one call.
        layers: dict = {}
        off = 0
        for name, p in self.module.named_parameters():
            if not p.requires_grad:
                continue
            m = re.search(r"_l(\d+)", name)
            key = int(m.group(1)) if m else -1
            lo, hi, ps = layers.get(key, (off, off, []))
            if hi != off:
                return  # not contiguous
            layers[key] = (lo, off + p.numel(), ps + [p])
            off += p.numel()
        if len(layers) < 2:
            return
        for b, (lo, hi, ps) in enumerate(layers.values()):
            self._buckets.append((lo, hi, len(ps)))
            for p in ps:
                p.register_post_accumulate_grad_hook(lambda _p, b=b: self._param_ready(b))
        self._pending = [n for _, _, n in self._buckets]
        self.overlap_active = True

    def _param_ready(self, b: int) -> None:
        if not self._in_step or not self.overlap_active:
            return  # a backward outside step(), or overlap off: leave the gradients alone
        self._pending[b] -= 1
        if self._pending[b] == 0:
            lo, hi, _ = self._buckets[b]
            self._works.append(
                dist.all_reduce(self.grad[lo:hi], op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def loss(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        out, _ = self.module(x)
        if out.is_cuda and out.dtype == torch.float32 and not target.requires_grad:
            return mse_loss(out, target)  # the library's one-pass loss and gradient
        return F.mse_loss(out, target)  # CPU ranks (gloo tests with torch.nn.GRU)

    def step(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One train step on this rank's shard; returns the shard loss (detached)."""
        loss = self.forward_backward(x, target)
        self.reduce_and_update()
        return loss

    def forward_backward(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """Zero the gradients, forward, loss and backward (the per-layer
        all-reduces start here when bucket overlap is on)."""
        self.grad.zero_()
        if self.overlap_active:
            self._pending = [n for _, _, n in self._buckets]
            self._works = []
        loss = self.loss(x, target)
        self._in_step = True
        try:
            loss.backward()
        finally:
            self._in_step = False
        return loss.detach()

    def reduce_and_update(self) -> None:
        """Finish the gradient all-reduce and apply the SGD update."""
        if self.world > 1 and self.overlap_active:
            for w in self._works:
                w.wait()
            # a layer whose parameters got no gradient this step
            for (lo, hi, _), left in zip(self._buckets, self._pending):
                if left > 0:
                    dist.all_reduce(self.grad[lo:hi], op=dist.ReduceOp.SUM, group=self.group)
            self._works = []
        elif self.world > 1:
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM, group=self.group)
        with torch.no_grad():
            self.flat.add_(self.grad, alpha=-self.lr / self.world)


class GraphedTrainStep:
    """A :class:`DataParallelTrainer` step replayed from CUDA graphs.

    The device work of zeroing the gradients, the forward, the loss and the
    backward (this library's kernels and torch's) is captured once per static
    input pair and replayed with one launch.  With ``include_update`` the
    gradient all-reduce (NCCL, captured into the graph) and the SGD update
    are part of the same graph, so a whole train step is one launch and no
    host work sits between its kernels; otherwise they run eagerly after each
    replay.  ``include_update`` is meant for a single process: capturing the
    NCCL all-reduce was measured to hang a 2-process run here, so with a
    process group keep the all-reduce eager.
    ``inputs`` lists the static ``(x, target)`` device tensor pairs (for
    instance the two buffer sets of a :class:`HostBatchPrefetcher`);
    ``step(i)`` replays graph ``i`` on whatever those tensors hold now.
    Per-layer bucket overlap is switched off for the trainer (its hooks
    stay registered but do nothing; the all-reduce of the whole buffer
    follows the replay); ``close()`` switches it back on.  Capture warms up on a side stream first (``warmup`` steps per
    input pair), as CUDA graph capture requires; those warm-up steps train
    like any other step.  ``capture_error_mode`` is passed to
    ``torch.cuda.graph``; with a process group, "thread_local" keeps other
    threads (NCCL's watchdog) free to query CUDA while this one captures.
    """

    def __init__(self, trainer: DataParallelTrainer, inputs, warmup: int = 3,
                 capture_error_mode: str = "global", include_update: bool = False) -> None:
        if include_update and trainer.world > 1:
            raise ValueError("GraphedTrainStep(include_update=True) is for a single process: keep the NCCL "
                             "all-reduce eager with a process group")
        self.trainer = trainer
        self.include_update = include_update
        trainer.overlap_active = False
        trainer._pending = [n for _, _, n in trainer._buckets]
        trainer._works = []
        self.inputs = list(inputs)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                for x, y in self.inputs:
                    trainer.step(x, y)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graphs, self.losses = [], []
        for x, y in self.inputs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode=capture_error_mode):
                loss = trainer.forward_backward(x, y)
                if include_update:
                    trainer.reduce_and_update()
            self.graphs.append(g)
            self.losses.append(loss)

    def step(self, i: int = 0) -> torch.Tensor:
        self.graphs[i].replay()
        if not self.include_update:
            self.trainer.reduce_and_update()
        return self.losses[i]

    def close(self) -> None:
        """Drop the graphs and give the trainer its per-layer overlap back."""
        self.graphs, self.losses = [], []
        self.trainer.overlap_active = bool(self.trainer._buckets) and self.trainer.world > 1


class HostBatchPrefetcher:
    """Double-buffered host-to-device staging of training batches.

    ``put(*host_tensors)`` starts copying one batch (pinned host tensors, for
    truly asynchronous copies) into the idle one of two device buffer sets, on
    a dedicated copy stream; ``get()`` makes the current (compute) stream wait
    for the oldest outstanding copy and returns its device tensors.  Calling
    ``put`` for batch k+1 right after ``get`` for batch k overlaps that copy
    with step k's kernels, as a pinned-memory data loader does.

    A buffer set is refilled only after the compute stream has finished the
    step that read it: ``get`` records that point (after the previous step's
    work was enqueued) and ``put`` makes the copy stream wait for it.
    """

    def __init__(self, device: torch.device, copy_stream: Optional[torch.cuda.Stream] = None) -> None:
        self.device = torch.device(device)
        self.stream = copy_stream if copy_stream is not None else torch.cuda.Stream(self.device)
        self._bufs: list = [None, None]
        self._ready: list = [None, None]
        self._free: list = [None, None]
        self._fill = 0          # slot the next put() fills
        self._queue: list = []  # slots filled, not yet handed out
        self._in_use: Optional[int] = None

    def put(self, *host: torch.Tensor) -> None:
        if len(self._queue) >= 2:
            raise RuntimeError("HostBatchPrefetcher holds two batches already; call get() first")
        slot = self._fill
        self._fill ^= 1
        bufs = self._bufs[slot]
        if bufs is None or len(bufs) != len(host) or any(
                b.shape != h.shape or b.dtype != h.dtype for b, h in zip(bufs, host)):
            # allocated on the current stream and kept for the object's lifetime
            bufs = tuple(torch.empty(h.shape, dtype=h.dtype, device=self.device) for h in host)
            self._bufs[slot] = bufs
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            if self._free[slot] is not None:
                self.stream.wait_event(self._free[slot])
            for d, h in zip(bufs, host):
                d.copy_(h, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self._ready[slot] = ev
        self._queue.append(slot)

    def get(self):
        if not self._queue:
            raise RuntimeError("HostBatchPrefetcher.get() without a pending put()")
        cur = torch.cuda.current_stream(self.device)
        if self._in_use is not None:
            # everything enqueued so far (the previous step) has read that slot
            ev = torch.cuda.Event()
            ev.record(cur)
            self._free[self._in_use] = ev
        slot = self._queue.pop(0)
        cur.wait_event(self._ready[slot])
        self._in_use = slot
        bufs = self._bufs[slot]
        return bufs if len(bufs) != 1 else bufs[0]
