"""The NumPy oracle against the golden fixtures made from the reference's own
CustomGRU (src/rnn_kernel/custom_gru.py) and torch.nn.GRU, and against
torch.nn.GRU directly on random shapes.  CPU only."""
import numpy as np
import pytest
import torch

from oracle import gru_oracle as O
from tests import golden_io


def _run_oracle(d, dtype):
    x = d["x"].astype(dtype)
    h0 = d["h0"].astype(dtype)
    ps = golden_io.params(d, dtype)
    out, hn, saved = O.gru_forward(x, h0, ps)
    if d["mse"]:
        tgt = d["target"].astype(dtype)
        dout = (2.0 / out.size) * (out - tgt)
        dout = dout.astype(dtype)
        dhn = None
    else:
        dout = d["grad_out"].astype(dtype)
        dhn = d["grad_h"].astype(dtype)
    dx, dh0, grads = O.gru_backward(dout, dhn, ps, saved)
    res = {"out": out, "hn": hn, "dx": dx, "dh0": dh0}
    for l, g in enumerate(grads):
        res[f"dweight_ih_l{l}"] = g["dw_ih"]
        res[f"dweight_hh_l{l}"] = g["dw_hh"]
        res[f"dbias_ih_l{l}"] = g["db_ih"]
        res[f"dbias_hh_l{l}"] = g["db_hh"]
    return res


@pytest.mark.parametrize("case", golden_io.CASES)
def test_oracle_fp64_matches_reference_customgru(case):
    d = golden_io.load(case)
    res = _run_oracle(d, np.float64)
    for k, v in res.items():
        np.testing.assert_allclose(v, d[f"custom64_{k}"], rtol=1e-10, atol=1e-12, err_msg=k)


@pytest.mark.parametrize("case", golden_io.CASES)
def test_oracle_fp32_matches_torch_gru_fp32(case):
    d = golden_io.load(case)
    res = _run_oracle(d, np.float32)
    for k, v in res.items():
        np.testing.assert_allclose(v, d[f"torch32_{k}"], rtol=1e-4, atol=1e-5, err_msg=k)


def test_golden_reference_customgru_fp32_matches_torch():
    # Pins the fixtures themselves: the reference's CustomGRU in FP32 agrees
    # with torch.nn.GRU to 1e-6 (tests/test_custom_gru.py:126-127 tolerance).
    for case in ("smoke", "h7_l2", "h33"):
        d = golden_io.load(case)
        for k in [k for k in d if k.startswith("custom32_")]:
            np.testing.assert_allclose(d[k], d["torch32_" + k[len("custom32_"):]], rtol=1e-5, atol=1e-6, err_msg=k)


@pytest.mark.parametrize("H,I,L", [(1, 1, 1), (5, 3, 3), (40, 17, 2)])
def test_oracle_matches_torch_gru_random(H, I, L):
    torch.manual_seed(H * 100 + I)
    B, T = 3, 7
    g = torch.nn.GRU(I, H, num_layers=L, batch_first=True).double()
    x = torch.randn(B, T, I, dtype=torch.float64, requires_grad=True)
    h0 = torch.randn(L, B, H, dtype=torch.float64, requires_grad=True)
    out, hn = g(x, h0)
    go, gh = torch.randn_like(out), torch.randn_like(hn)
    torch.autograd.backward([out, hn], [go, gh])
    ps = [tuple(getattr(g, f"{p}_l{l}").detach().numpy() for p in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"))
          for l in range(L)]
    o_out, o_hn, saved = O.gru_forward(x.detach().numpy(), h0.detach().numpy(), ps)
    np.testing.assert_allclose(o_out, out.detach().numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(o_hn, hn.detach().numpy(), rtol=1e-10, atol=1e-12)
    dx, dh0, grads = O.gru_backward(go.numpy(), gh.numpy(), ps, saved)
    np.testing.assert_allclose(dx, x.grad.numpy(), rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(dh0, h0.grad.numpy(), rtol=1e-9, atol=1e-11)
    for l in range(L):
        np.testing.assert_allclose(grads[l]["dw_ih"], g.__getattr__(f"weight_ih_l{l}").grad.numpy(), rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose(grads[l]["dw_hh"], g.__getattr__(f"weight_hh_l{l}").grad.numpy(), rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose(grads[l]["db_ih"], g.__getattr__(f"bias_ih_l{l}").grad.numpy(), rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose(grads[l]["db_hh"], g.__getattr__(f"bias_hh_l{l}").grad.numpy(), rtol=1e-9, atol=1e-11)


def test_oracle_empty_sequence():
    B, I, H = 2, 3, 4
    rng = np.random.default_rng(0)
    ps = (rng.standard_normal((3 * H, I)), rng.standard_normal((3 * H, H)),
          rng.standard_normal(3 * H), rng.standard_normal(3 * H))
    x = np.zeros((B, 0, I))
    h0 = rng.standard_normal((B, H))
    out, hn, st = O.gru_layer_forward(x, h0, *ps)
    assert out.shape == (B, 0, H)
    np.testing.assert_array_equal(hn, h0)
    dhn = rng.standard_normal((B, H))
    res = O.gru_layer_backward(None, dhn, x, ps[0], ps[1], st)
    np.testing.assert_array_equal(res["dh0"], dhn)
    assert not res["dw_hh"].any()
