"""Generate the golden GRU fixtures in this folder.

Run in a checkout that has the reference repository (HanXuxx/RNN_kernel)
available; pass its root with ``--reference``.  The script imports the
reference's pure-torch ``CustomGRU`` (``src/rnn_kernel/custom_gru.py``) and
runs it, in float32 and float64, together with ``torch.nn.GRU`` float32 on
the same seeded inputs, and stores inputs, outputs and every gradient.

Cases mirror the reference's own parity tests:

* ``smoke``       - the quick-check shape (I=H=16, B=2, T=8, seed 0,
                    h0=0, MSE against an N(0,1) target);
* ``h7_l2``       - ``tests/test_custom_gru.py:17-22`` (seed 321, I=4, H=7, L=2,
                    B=3, T=5, random h0, random grad_out / grad_h);
* ``h33`` / ``h130`` / ``h129``  - odd hidden sizes (``tests/test_a100_gru_forward.py``
                    uses H in {16,33,128,130,160,256});
* ``h256``        - ``tests/test_a100_prod.py:84-126`` shape (H=256, I=16, L=1,
                    B=2, seed 2130 + 10*L + I; T=4 keeps the file small).

The float32 CustomGRU results are stored only for H <= 33 (they are FP32 noise
around the float64 ones and would dominate the file size at large H).

The fixtures are plain ``.npz`` files; nothing at test time needs the
reference repository.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = {
    # name: (seed, I, H, L, B, T, loss)
    "smoke": (0, 16, 16, 1, 2, 8, "mse"),
    "h7_l2": (321, 4, 7, 2, 3, 5, "random"),
    "h33": (33, 5, 33, 1, 3, 6, "random"),
    "h129": (129, 7, 129, 1, 2, 5, "random"),
    "h130": (130, 16, 130, 1, 2, 5, "random"),
    "h256": (2130 + 10 + 16, 16, 256, 1, 2, 4, "random"),
}


def run_case(CustomGRU, copy_from_torch_gru, name, seed, I, H, L, B, T, loss):
    torch.manual_seed(seed)
    ref = torch.nn.GRU(I, H, num_layers=L, batch_first=True)
    x = torch.randn(B, T, I)
    if loss == "mse":
        h0 = torch.zeros(L, B, H)
        target = torch.randn(B, T, H)
        grad_out = grad_h = None
    else:
        h0 = torch.randn(L, B, H)
        target = None
        grad_out = torch.randn(B, T, H)
        grad_h = torch.randn(L, B, H)

    results = {}

    def run(model, dtype, tag):
        m = model.to(dtype)
        xx = x.to(dtype).clone().requires_grad_(True)
        hh = h0.to(dtype).clone().requires_grad_(True)
        out, hn = m(xx, hh)
        if loss == "mse":
            lv = torch.nn.functional.mse_loss(out, target.to(dtype))
            lv.backward()
            results[f"{tag}_loss"] = lv.detach().double().numpy()
        else:
            out.backward(grad_out.to(dtype), retain_graph=True)
            hn.backward(grad_h.to(dtype))
        results[f"{tag}_out"] = out.detach().double().numpy()
        results[f"{tag}_hn"] = hn.detach().double().numpy()
        results[f"{tag}_dx"] = xx.grad.double().numpy()
        results[f"{tag}_dh0"] = hh.grad.double().numpy()
        for l in range(L):
            for p in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
                results[f"{tag}_d{p}_l{l}"] = getattr(m, f"{p}_l{l}").grad.double().numpy()

    for dtype, tag in ((torch.float32, "custom32"), (torch.float64, "custom64")):
        cg = CustomGRU(I, H, L, pointwise_backend="torch", batch_first=True)
        copy_from_torch_gru(cg, ref)
        run(cg, dtype, tag)
    ref32 = torch.nn.GRU(I, H, num_layers=L, batch_first=True)
    ref32.load_state_dict(ref.state_dict())
    run(ref32, torch.float32, "torch32")

    arrays = {
        "meta": np.array([seed, I, H, L, B, T, 1 if loss == "mse" else 0], np.int64),
        "x": x.numpy(),
        "h0": h0.numpy(),
    }
    if target is not None:
        arrays["target"] = target.numpy()
    else:
        arrays["grad_out"] = grad_out.numpy()
        arrays["grad_h"] = grad_h.numpy()
    for l in range(L):
        for p in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
            arrays[f"{p}_l{l}"] = getattr(ref, f"{p}_l{l}").detach().numpy()
    for k, v in results.items():
        if k.startswith("custom32") and H > 33:
            continue
        arrays[k] = v if k.startswith("custom64") else v.astype(np.float32)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from rnn_kernel.custom_gru import CustomGRU, copy_from_torch_gru  # noqa: E402

    torch.set_num_threads(1)
    for name, spec in CASES.items():
        run_case(CustomGRU, copy_from_torch_gru, name, *spec)


if __name__ == "__main__":
    main()
