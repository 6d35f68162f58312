#!/usr/bin/env python
"""GRU FP32 train-step benchmark (samples*timesteps/s).

One step = forward + MSE loss + backward + (all-reduce for N > 1) + SGD
lr 1e-2 of a 1-layer GRU, I = H = 256, T = 512, batch 64 per GPU (the
reference's production a100_gru_h256 shape at N = 1; weak scaling at N > 1:
the data-parallel step with 64 rows per rank).  ``--global-batch`` switches
the headline to strong scaling (a global batch split evenly over the ranks).

Beside the headline the line carries
* ``strong``: the data-parallel workload with a global batch of 1024 split
  evenly over the N ranks (I = H = 256, T = 512), timed the same way;
* ``dp_check`` (N > 1): 10 data-parallel steps on that workload (rank r
  draws its shard from seed + r) against one GPU running the concatenated
  batch from the same initial weights: loss and weights must agree;
* ``cudnn_sweep`` (N = 1): this library vs cuDNN ``torch.nn.GRU`` on the
  same GPU over hidden sizes 64..256 (I = H, B = 64, T = 256), the stacked
  2-layer shape (I = 128, H = 256, B = 128, T = 1024, loss sum(out^2),
  random h0) and the B = 1024 batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N

Rank 0 prints one JSON line.  Timing: W untimed warm-up steps, then exactly K
steps, each bracketed by CUDA events on the launching stream, with a 256 MiB
L2 flush between steps outside the events; barrier + synchronize on both
sides; per-step statistics are the max over ranks.  A ~30 ms device sleep
before the first timed step lets the host enqueue ahead of the GPU.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GRU fp32 train samples·timesteps/s at H=256, 1/2/4/8 B200 vs cuDNN & host CPU"
UNIT = "samples*timesteps/s"
STRONG_GLOBAL_BATCH = 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch-per-gpu", type=int, default=64)
    ap.add_argument("--global-batch", type=int, default=0, help="strong scaling: split this batch over ranks")
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--input-size", type=int, default=256)
    ap.add_argument("--hidden-size", type=int, default=256)
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cudnn", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-strong", action="store_true", help="skip the global-batch-1024 sub-measurement")
    ap.add_argument("--no-dp-check", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the cuDNN comparison sweep")
    ap.add_argument("--no-graph", action="store_true", help="eager steps only (no CUDA graph replay)")
    ap.add_argument("--timeline", action="store_true",
                    help="profiling only: use the instrumented library build and add the time loops' per-phase "
                         "step timeline (clock64 cycles) to the line; its step times are not bench values")
    ap.add_argument("--time-chunks", type=int, default=0,
                    help="time chunks of the forward/backward (0 automatic, 1 off, 2..4 forced where possible)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and throttle reasons of one GPU, sampled every few ms
    through NVML on a thread (nvidia-smi's polling is too coarse for a timed
    region of tens of milliseconds); one nvidia-smi reading when NVML is
    unavailable.  Reads settings only; changes nothing."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.rows = []  # (sm_mhz, max_mhz, power_w, [reason flags])
        self.error = None
        self._stop = threading.Event()
        self._thr = None
        self._nv = None
        self._h = None

    def _handle(self):
        import pynvml as nv

        nv.nvmlInit()
        self._nv = nv
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
            return nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def _sample(self):
        nv, h = self._nv, self._h
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        flags = [bool(rs & nv.nvmlClocksEventReasonHwSlowdown),
                 bool(rs & nv.nvmlClocksEventReasonHwThermalSlowdown),
                 bool(rs & nv.nvmlClocksEventReasonSwThermalSlowdown),
                 bool(rs & nv.nvmlClocksEventReasonSwPowerCap)]
        self.rows.append((float(sm), float(mx), pw, flags))

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception as exc:  # pragma: no cover - depends on the driver
                self.error = f"{type(exc).__name__}: {exc}"
                return
            time.sleep(self.period)

    def __enter__(self):
        try:
            self._h = self._handle()
            self._sample()  # live before the timed region starts
        except Exception as exc:
            self._h = None
            self.error = f"NVML unavailable: {type(exc).__name__}: {exc}"
            return self
        self._thr = threading.Thread(target=self._loop, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=5)
        if self._h is None:
            self.rows = nvidia_smi_sample(self.cuda_index)

    def summary(self):
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "error": self.error}
        load = [r for r in rows if r[2] > 200.0] or rows
        sm = sorted(r[0] for r in load)
        reasons = sorted({n for r in load for n, f in zip(self.NAMES, r[3]) if f})
        out = {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
               "samples": len(load), "power_w_max": max(r[2] for r in rows),
               "source": "nvml" if self._h is not None else "nvidia-smi"}
        if self.error:
            out["error"] = self.error
        return out


def nvidia_smi_sample(gpu: int):
    q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=20).stdout
    except (OSError, subprocess.SubprocessError):
        return []
    rows = []
    for line in out.splitlines():
        p = [x.strip() for x in line.split(",")]
        try:
            rows.append((float(p[0]), float(p[1]), float(p[2]), [v.lower().startswith("active") for v in p[3:7]]))
        except (ValueError, IndexError):
            continue
    return rows


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU implementation of the path
# ---------------------------------------------------------------------------
def run_reference(args, world, rank):
    if rank != 0:
        return 0
    from oracle.cpu_baseline import time_cpu_train_step

    # The whole job's batch (all ranks' shards), run on the host cores.
    B = args.global_batch if args.global_batch else args.batch_per_gpu * world
    T, I, H = args.seq_len, args.input_size, args.hidden_size
    # One step of the full workload takes about a second on a many-core host;
    # cap the count so the whole run stays within a few minutes.
    steps = max(1, min(args.steps, 10))
    warm = max(1, min(args.warmup, 2))
    r = time_cpu_train_step(B, T, I, H, warmup=warm, steps=steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic N(0,1) x and target",
        "config": {"workload": f"gru_train_step I={I} H={H} T={T}, global batch {B} on the host CPU",
                   "global_batch": B,
                   "seq_len": T, "input_size": I, "hidden_size": H, "layers": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                         "sample": f"torch.nn.GRU FP32 train step on host CPU ({r['cpu_model']}), "
                                   f"full global B={B},T={T}, {warm} warm-up + {steps} timed steps"},
        "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# roofline bookkeeping
# ---------------------------------------------------------------------------
def fp32_peak_tflops(sm_mhz: float, sms: int = 148) -> float:
    # 128 FP32 FMA lanes per SM, 2 FLOP per FMA.
    return sms * 128 * 2 * sm_mhz * 1e6 / 1e12


def recurrent_flops(b, T, H, bwd: bool) -> float:
    # per timestep: the b x 3H x H recurrent product + the gate arithmetic
    # (10 FLOP per element forward, 16 backward; transcendental = 1).
    return T * (2.0 * b * 3 * H * H + (16 if bwd else 10) * b * H)


def step_roofline_ms(b, T, H, sm_mhz: float, sms: int = 148) -> float:
    p_fp32 = fp32_peak_tflops(sm_mhz, sms) * 1e12
    bw_smem = sms * 128 * sm_mhz * 1e6  # bytes/s
    w_bytes = 3 * H * H * 4
    t_f = w_bytes / bw_smem + (2 * b * 3 * H * H + 10 * b * H) / p_fp32
    t_b = w_bytes / bw_smem + (2 * b * 3 * H * H + 16 * b * H) / p_fp32
    return 1e3 * T * (t_f + t_b)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


def load_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
# Set in main() when several ranks run: a tiny all-reduce that lines the
# ranks' GPUs up after the pre-timing device sleep (outside every event
# window).  Without it, a rank whose host reached the timed region later (rank
# 0 waits for its clock sampler's first sample) made the first all-reduce of
# the other ranks wait for it inside their first timed step.
ALIGN_RANKS = None


def timed_steps(step_fn, K, flush, torch):
    """Per-step device times (ms).  A device-side sleep first lets the host
    enqueue the K steps ahead of the GPU, so a host-side stall while
    launching (seen at 8 ranks: one step in 20 waiting 10-18 ms for its
    launches) does not leave the GPU idle inside a step's event window; the
    sleep itself is outside every window."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    sleep = getattr(torch.cuda, "_sleep", None)
    if sleep is not None:
        sleep(int(30e-3 * 1.965e9))  # ~30 ms of device cycles
    if ALIGN_RANKS is not None:
        ALIGN_RANKS()
    for k in range(K):
        flush()
        evs[k][0].record()
        step_fn(k)
        evs[k][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def step_timeline(lib):
    """Per-phase cycles of the time loops from the instrumented build: for each
    loop, CTA 0 / thread 0 (which has a pointwise item) and CTA 0's last
    thread (an input-prefetch issuer when the last sub-chunk leaves threads
    idle), the median over 8 consecutive steps of each point's clock64 offset
    from the step start, and the median step length in cycles."""
    import numpy as np

    buf = lib.timeline_read()
    out = {"source": "clock64 at marked points of steps 100-107 of the last launch of each loop "
                     "(instrumented build, RNN_KERNEL_B200_VARIANT=timeline)"}
    for d, name in enumerate(("fwd", "bwd")):
        pts = lib.TIMELINE_POINTS[name]
        rec = {}
        for w, who in ((0, "cta0_thread0"), (1, "cta0_last_thread")):
            tl = buf[d, w]
            steps = np.diff(tl[:, 0])
            ph = {}
            for k, pn in enumerate(pts):
                col = tl[:, k]
                if np.all(col != 0):
                    ph[pn] = int(np.median(col - tl[:, 0]))
            rec[who] = {"step_cycles": int(np.median(steps)) if len(steps) else None, "offsets": ph}
        out[name] = rec
    return out


def step_stats(times, world, dev, torch, dist):
    """mean / p50 / p90 / max of per-step ms, each the max over ranks."""
    srt = sorted(times)
    n = len(srt)

    def pct(q):
        return srt[min(n - 1, max(0, int(round(q * (n - 1)))))]

    v = [sum(times) / n, pct(0.5), pct(0.9), srt[-1]]
    if world > 1:
        t = torch.tensor(v, device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        v = [float(x) for x in t]
    return {"mean": v[0], "p50": v[1], "p90": v[2], "max": v[3]}


# ---------------------------------------------------------------------------
# sub-measurements
# ---------------------------------------------------------------------------
def strong_scaling(args, world, rank, dev, K, W, flush, barrier, torch, dist):
    """Global batch 1024 split over the ranks (I = H = 256, T = 512)."""
    from rnn_kernel_b200 import GRU, DataParallelTrainer, GraphedTrainStep

    Bg, T, I, H = STRONG_GLOBAL_BATCH, 512, 256, 256
    b = Bg // world
    torch.manual_seed(0)
    model = GRU(I, H).to(dev)
    trainer = DataParallelTrainer(model, lr=1e-2)
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    x = torch.randn(b, T, I, device=dev, generator=g)
    y = torch.randn(b, T, H, device=dev, generator=g)
    for _ in range(W):
        trainer.step(x, y)
    graph = None
    if not args.no_graph:
        graph = GraphedTrainStep(trainer, [(x, y)], warmup=1,
                                 capture_error_mode="thread_local" if world > 1 else "global",
                                 include_update=world == 1)
        for _ in range(W):  # untimed replays (the first one uploads the graph)
            graph.step(0)
    barrier()
    torch.cuda.synchronize()
    times = timed_steps((lambda k: graph.step(0)) if graph else (lambda k: trainer.step(x, y)), K, flush, torch)
    barrier()
    st = step_stats(times, world, dev, torch, dist)
    out = {"global_batch": Bg, "batch_per_gpu": b, "seq_len": T, "input_size": I, "hidden_size": H,
           "scaling": "strong", "value": Bg * T / (st["mean"] / 1e3), "unit": UNIT,
           "ms_per_step": st["mean"], "p50_ms": st["p50"], "p90_ms": st["p90"], "max_ms": st["max"],
           "graph": graph is not None}
    del graph, trainer, model, x, y
    torch.cuda.empty_cache()
    return out


def dp_equivalence(world, rank, dev, barrier, torch, dist, steps=10):
    """10 data-parallel steps (global batch 1024 split over the ranks, rank r's
    shard from seed + r) against one GPU running the concatenated batch from
    the same initial weights."""
    from rnn_kernel_b200 import GRU, DataParallelTrainer

    Bg, T, I, H, lr, seed = STRONG_GLOBAL_BATCH, 512, 256, 256, 1e-2, 3000
    b = Bg // world
    solo = dist.new_group([0])  # collective: every rank creates it

    def shard(r, step):
        g = torch.Generator(device=dev).manual_seed(seed + r + 1000 * step)
        return (torch.randn(b, T, I, device=dev, generator=g), torch.randn(b, T, H, device=dev, generator=g))

    torch.manual_seed(0)
    model = GRU(I, H).to(dev)
    tr = DataParallelTrainer(model, lr=lr)
    init = tr.flat.detach().clone()
    losses = []
    for step in range(steps):
        x, y = shard(rank, step)
        loss = tr.step(x, y)
        dist.all_reduce(loss)
        losses.append(float(loss) / world)
    barrier()
    res = None
    if rank == 0:
        m1 = GRU(I, H).to(dev)
        t1 = DataParallelTrainer(m1, lr=lr, process_group=solo)
        with torch.no_grad():
            t1.flat.copy_(init)
        l1 = []
        for step in range(steps):
            xs, ys = zip(*[shard(r, step) for r in range(world)])
            l1.append(float(t1.step(torch.cat(xs), torch.cat(ys))))
        a, r_ = tr.flat.double(), t1.flat.double()
        diff = (a - r_).abs()
        lim = 1e-5 + 1e-4 * r_.abs()
        loss_rel = max(abs(p - q) / abs(q) for p, q in zip(losses, l1))
        res = {"steps": steps, "global_batch": Bg, "max_abs_weight_diff": float(diff.max()),
               "worst_ratio_to_tol": float((diff / lim).max()), "loss_rel_diff": loss_rel,
               "final_loss": l1[-1], "tolerance": "weights rtol 1e-4 / atol 1e-5 element-wise; loss rel 1e-4",
               "pass": bool((diff <= lim).all()) and loss_rel <= 1e-4}
        del t1, m1
    barrier()
    del tr, model
    torch.cuda.empty_cache()
    return res


def cudnn_sweep(W, K, flush, torch):
    """This library vs cuDNN torch.nn.GRU (TF32 off) on the same GPU, same
    step (forward + loss + backward + SGD), median ms of K steps each."""
    from torch import nn

    from rnn_kernel_b200 import GRU

    dev = torch.device("cuda", torch.cuda.current_device())
    cases = [dict(name=f"H{h}", I=h, H=h, B=64, T=256, L=1, loss="mse", h0=0.0)
             for h in (64, 96, 128, 129, 130, 160, 192, 256)]
    cases.append(dict(name="stacked_L2_I128_H256_B128_T1024", I=128, H=256, B=128, T=1024, L=2, loss="sumsq",
                      h0=0.1))
    cases.append(dict(name="B1024_I256_H256_T512", I=256, H=256, B=1024, T=512, L=1, loss="mse", h0=0.0))
    out = []
    for c in cases:
        I, H, B, T, L = c["I"], c["H"], c["B"], c["T"], c["L"]
        g = torch.Generator(device=dev).manual_seed(H)
        x = torch.randn(B, T, I, device=dev, generator=g)
        y = torch.randn(B, T, H, device=dev, generator=g)
        h0 = c["h0"] * torch.randn(L, B, H, device=dev, generator=g)

        def lossf(o, c=c, y=y):
            return torch.nn.functional.mse_loss(o, y) if c["loss"] == "mse" else (o * o).sum()

        torch.manual_seed(H)
        ours = GRU(I, H, num_layers=L).to(dev)
        ref = nn.GRU(I, H, num_layers=L, batch_first=True).to(dev)
        with torch.no_grad():
            for p, q in zip(ref.parameters(), ours.parameters()):
                p.copy_(q)
        ref.flatten_parameters()
        res = {"case": c["name"], "I": I, "H": H, "B": B, "T": T, "layers": L}
        for tag, m in (("ours", ours), ("cudnn", ref)):
            opt = torch.optim.SGD(m.parameters(), lr=1e-2)

            def step(k, m=m, opt=opt, x=x, h0=h0, lossf=lossf):
                opt.zero_grad(set_to_none=True)
                o, _ = m(x, h0)
                lossf(o).backward()
                opt.step()

            for _ in range(W):
                step(0)
            torch.cuda.synchronize()
            ts = sorted(timed_steps(step, K, flush, torch))
            res[f"{tag}_ms"] = ts[len(ts) // 2]
            del opt
        res["speedup"] = res["cudnn_ms"] / res["ours_ms"]
        out.append(res)
        del ours, ref, x, y, h0
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    if args.timeline:  # before the package is imported: it picks its library at import
        os.environ["RNN_KERNEL_B200_VARIANT"] = "timeline"
    import torch
    import torch.distributed as dist

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
        global ALIGN_RANKS
        _align = torch.zeros(1, device=dev)
        ALIGN_RANKS = lambda: dist.all_reduce(_align)  # noqa: E731

    from rnn_kernel_b200 import GRU, DataParallelTrainer, GraphedTrainStep, _lib

    _lib.set_time_chunks(args.time_chunks)
    B = args.global_batch // world if args.global_batch else args.batch_per_gpu
    T, I, H, L = args.seq_len, args.input_size, args.hidden_size, args.layers
    K, W = args.steps, max(3, args.warmup)
    scaling = "strong" if args.global_batch else "weak"

    torch.manual_seed(0)
    model = GRU(I, H, num_layers=L).to(dev)
    trainer = DataParallelTrainer(model, lr=1e-2)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(B, T, I, device=dev, generator=g)
    y = torch.randn(B, T, H, device=dev, generator=g)
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, device=dev)

    def flush():
        flush_buf.zero_()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(W):
        trainer.step(x, y)
    torch.cuda.synchronize()

    # ---- eager pass: per-kernel device times (library telemetry) ----
    barrier()
    torch.cuda.synchronize()
    _lib.timing_enable(True)
    _lib.timing_collect()
    launches0 = _lib.launch_count()
    etimes = timed_steps(lambda k: trainer.step(x, y), K, flush, torch)
    launches_eager = _lib.launch_count() - launches0
    _lib.timing_enable(False)
    ktimes = _lib.timing_collect()
    torch.cuda.synchronize()
    barrier()
    est = step_stats(etimes, world, dev, torch, dist)
    timeline = step_timeline(_lib) if args.timeline else None

    # ---- headline: the same step replayed from a CUDA graph ----
    # (zero grads + fwd + loss + bwd captured, and at N = 1 the SGD update
    # too: one launch per step; at N > 1 the NCCL all-reduce and the update
    # run eagerly after the replay).  Library kernels per replay = launches
    # during capture.
    graph, graph_error, per_step_lib = None, None, 0
    cmode = "thread_local" if world > 1 else "global"
    if not args.no_graph:
        try:
            n0 = _lib.launch_count()
            graph = GraphedTrainStep(trainer, [(x, y)], warmup=3, capture_error_mode=cmode,
                                     include_update=world == 1)
            per_step_lib = (_lib.launch_count() - n0) - 3 * (launches_eager // K)
        except Exception as exc:  # capture unavailable: eager headline
            graph = None
            graph_error = f"{type(exc).__name__}: {exc}"[:200]
    graphed = graph is not None
    if graph is not None:
        # untimed replays: the first launch of an instantiated graph uploads it
        for _ in range(W):
            graph.step(0)
    barrier()
    torch.cuda.synchronize()
    # only rank 0 reports clocks: the other ranks do not poll NVML (8 processes
    # polling the driver at once stalled host threads)
    with (ClockSampler(local) if rank == 0 else contextlib.nullcontext()) as clk:
        if graph is not None:
            times = timed_steps(lambda k: graph.step(0), K, flush, torch)
        else:
            times = timed_steps(lambda k: trainer.step(x, y), K, flush, torch)
    torch.cuda.synchronize()
    barrier()
    clocks = clk.summary() if rank == 0 else None
    st = step_stats(times, world, dev, torch, dist)
    ms = st["mean"]
    launches = per_step_lib * K if graph is not None else launches_eager
    value = B * world * T / (ms / 1e3)

    # ---- end to end through the public API from pinned host buffers ----
    # Every step copies its x and target from pinned host memory and reads the
    # loss back.  Headline: the copy of step k+1's batch runs on a copy stream
    # during step k (HostBatchPrefetcher, double-buffered), as a pinned-memory
    # data loader does; the timed region holds K copies and K steps.  Also
    # reported: the same loop with each copy issued serially before its step.
    e2e = None
    if not args.no_e2e:
        from rnn_kernel_b200 import HostBatchPrefetcher

        xh = x.cpu().pin_memory()
        yh = y.cpu().pin_memory()
        lh = torch.empty(1, pin_memory=True)

        # With the graph, each step replays the capture whose static inputs
        # are the buffers the batch was copied into.
        def e2e_serial_step(k):
            if graph is not None:
                x.copy_(xh, non_blocking=True)
                y.copy_(yh, non_blocking=True)
                loss = graph.step(0)
            else:
                xd = xh.to(dev, non_blocking=True)
                yd = yh.to(dev, non_blocking=True)
                loss = trainer.step(xd, yd)
            lh.copy_(loss.reshape(1), non_blocking=True)

        pf = HostBatchPrefetcher(dev)
        pgraph = None
        if graph is not None:
            # allocate both buffer sets, then capture one graph on each
            for _ in range(2):
                pf.put(xh, yh)
                pf.get()
            torch.cuda.synchronize()
            pgraph = GraphedTrainStep(trainer, [pf._bufs[0], pf._bufs[1]], warmup=1, capture_error_mode=cmode,
                                      include_update=world == 1)
            torch.cuda.synchronize()
        pf.put(xh, yh)  # one batch ahead from here on

        def e2e_step(k):
            xd, yd = pf.get()
            slot = pf._in_use
            pf.put(xh, yh)  # the next step's batch, into the other set, overlapped with this step
            loss = pgraph.step(slot) if pgraph is not None else trainer.step(xd, yd)
            lh.copy_(loss.reshape(1), non_blocking=True)

        def timed_e2e(fn):
            for _ in range(2):
                fn(0)
            torch.cuda.synchronize()
            barrier()
            return step_stats(timed_steps(fn, K, flush, torch), world, dev, torch, dist)

        serial = timed_e2e(e2e_serial_step)
        est2 = timed_e2e(e2e_step)
        while pf._queue:  # drain the outstanding prefetch
            pf.get()
        torch.cuda.synchronize()
        ems = est2["mean"]
        e2e = {"value": B * world * T / (ems / 1e3), "unit": UNIT, "ms_per_step": ems,
               "p50_ms": est2["p50"], "p90_ms": est2["p90"], "max_ms": est2["max"],
               "h2d_bytes_per_step": (x.numel() + y.numel()) * 4, "d2h_bytes_per_step": 4,
               "serial_ms_per_step": serial["mean"],
               "serial_value": B * world * T / (serial["mean"] / 1e3),
               "note": "per rank: x and target copied from pinned host memory and the loss copied back every step; "
                       "next step's copy overlapped with this step on a copy stream (HostBatchPrefetcher); "
                       "serial_*: each copy issued before its own step"}
        del pgraph, pf

    del graph
    torch.cuda.synchronize()

    # ---- strong scaling (global batch 1024) and the DP equivalence check ----
    strong = None if args.no_strong else strong_scaling(args, world, rank, dev, K, W, flush, barrier, torch, dist)
    dp_check = None
    if world > 1 and not args.no_dp_check:
        dp_check = dp_equivalence(world, rank, dev, barrier, torch, dist)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0
    ALIGN_RANKS = None  # rank 0 alone from here on (cuDNN and CPU comparisons)

    # ---- kernel roofline (dominant kernel, measured live in the timed region) ----
    per_kind = {k: {"ms_per_launch": (tot / n if n else None), "launches": n, "ms_per_step": tot / K}
                for k, (tot, n) in ktimes.items()}
    dom = max(("fwd_recurrent", "bwd_recurrent"), key=lambda k: ktimes[k][0])
    dom_ms = per_kind[dom]["ms_per_launch"]
    # with time chunks a layer's pass over the sequence is several launches,
    # each over T / chunks steps
    chunks = max(1, round(ktimes[dom][1] / (K * L))) if ktimes[dom][1] else 1
    flops = recurrent_flops(B, T, H, dom == "bwd_recurrent") / chunks
    achieved = flops / (dom_ms / 1e3) / 1e12 if dom_ms else None
    peak = fp32_peak_tflops(1965.0)
    roofline = {
        "bound": "fp32", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": (achieved / peak) if achieved else None, "traffic": load_traffic().get(dom),
        "traffic_source": "profiles/ncu_traffic.json: dram__bytes_read.sum + dram__bytes_write.sum of one "
                          "full-size launch from an ncu capture of the committed kernels (not measured in this run)",
        "peak_source": "nominal FP32 CUDA-core peak 148 SM x 128 FMA/clk x 2 x 1965 MHz "
                       "(MEASURED_PEAKS.json has HBM and bf16 tensor figures only)",
        "flops_per_launch": flops,
        "launches_per_pass": chunks,
        "us_per_timestep": dom_ms * 1e3 / (T / chunks) if dom_ms else None,
    }
    t_roof = step_roofline_ms(B, T, H, 1965.0) * L
    # Side-by-side bounds: + the step's tensor-core products at 3xTF32
    # (nominal 1.1 PFLOP/s TF32 / 3 passes), and the minimal HBM traffic of a
    # step (~(12 I + 132 H) bytes per sample-timestep per layer) at the
    # measured copy bandwidth.
    gemm_flop = 0.0
    for l in range(L):
        li = I if l == 0 else H
        n_prod = 3 if l == 0 else 4  # projection, dW_ih, dW_hh (+ dx into the layer below)
        gemm_flop += n_prod * 2.0 * B * T * 3 * H * li
    t_gemm = gemm_flop / (1.1e15 / 3) * 1e3
    hbm_gbs = measured_peaks().get("hbm_gbs") or 6650.0
    hbm_bytes = sum((12 * (I if l == 0 else H) + 132 * H) * B * T for l in range(L))
    step_roof = {"t_roof_ms": t_roof, "frac": t_roof / ms,
                 "definition": "T*(t_fwd+t_bwd), t = 3H^2*4B/SMEM_BW + (2*b*3H*H + {10|16}*b*H)/P_fp32, nominal peaks",
                 "full_step_bound_ms": t_roof + t_gemm, "full_step_frac": (t_roof + t_gemm) / ms,
                 "gemm_gflop_per_step": gemm_flop / 1e9,
                 "hbm_bound_ms": hbm_bytes / (hbm_gbs * 1e9) * 1e3, "hbm_bytes_per_step": hbm_bytes,
                 "hbm_peak_gbs": hbm_gbs}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms, "median_ms_per_step": st["p50"], "p90_ms_per_step": st["p90"],
        "max_ms_per_step": st["max"], "step_ms_rank0": [round(t, 4) for t in times], "higher_is_better": True,
        "graph": graphed, "eager_ms_per_step": est["mean"], "eager_median_ms_per_step": est["p50"],
        "scaling": scaling, "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic: x, target ~ N(0,1) per rank (seed 1000+rank); weights U(-1/16,1/16)",
        "config": {"workload": f"gru_train_step {L}-layer I={I} H={H} T={T}, batch {B}/GPU "
                               f"(fwd + MSE + bwd + allreduce + SGD lr 1e-2)",
                   "global_batch": B * world, "seq_len": T, "input_size": I, "hidden_size": H, "layers": L,
                   "parallelism": f"dp{world}", "l2": "256 MiB flush between timed steps (outside the events)",
                   "time_chunks": args.time_chunks},
        "clocks": clocks,
        "gpu_launches": int(launches),
        "kernels": per_kind,
        **({"timeline": timeline} if timeline is not None else {}),
        "roofline": roofline,
        "step_roofline": step_roof,
        "e2e": e2e,
        "strong": strong,
        "dp_check": dp_check,
        "impl": "b200",
    }
    if graph_error:
        line["graph_error"] = graph_error

    if world == 1 and not args.no_cudnn:
        from torch import nn

        torch.manual_seed(0)
        ref = nn.GRU(I, H, num_layers=L, batch_first=True).to(dev)
        ref.flatten_parameters()
        opt = torch.optim.SGD(ref.parameters(), lr=1e-2)

        def cudnn_step(k):
            opt.zero_grad(set_to_none=True)
            out, _ = ref(x)
            torch.nn.functional.mse_loss(out, y).backward()
            opt.step()

        for _ in range(W):
            cudnn_step(0)
        torch.cuda.synchronize()
        ct = timed_steps(cudnn_step, K, flush, torch)
        cms = sum(ct) / K
        line["cudnn"] = {"value": B * T / (cms / 1e3), "unit": UNIT, "ms_per_step": cms,
                         "what": "torch.nn.GRU (cuDNN, TF32 off) same step on the same GPU",
                         "speedup_of_b200": cms / ms}
        del opt, ref
        if not args.no_sweep:
            line["cudnn_sweep"] = cudnn_sweep(3, 7, flush, torch)

    if world == 1 and not args.no_cpu_baseline:
        from oracle.cpu_baseline import time_cpu_train_step

        r = time_cpu_train_step(B, T, I, H, warmup=1, steps=3)
        line["cpu_baseline"] = {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                                "sample": f"torch.nn.GRU FP32 train step on host CPU ({r['cpu_model']}), "
                                          f"full B={B},T={T} workload, 1 warm-up + 3 timed steps"}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
