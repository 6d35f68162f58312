"""Loading helpers for the fixtures in tests/golden (see make_golden.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ("smoke", "h7_l2", "h33", "h129", "h130", "h256")


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        d = {k: z[k] for k in z.files}
    seed, I, H, L, B, T, mse = (int(v) for v in d["meta"])
    d.update(seed=seed, I=I, H=H, L=L, B=B, T=T, mse=bool(mse))
    return d


def params(d: dict, dtype=np.float64):
    return [tuple(d[f"{p}_l{l}"].astype(dtype) for p in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"))
            for l in range(d["L"])]
