"""The C ABI called directly (ctypes, raw device pointers), checked against the
NumPy oracle -- the way a non-Python host would drive the library."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import gru_oracle as O
from rnn_kernel_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5


def _p(t):
    return None if t is None else t.data_ptr()


def _case(B, T, I, H, seed):
    rng = np.random.default_rng(seed)
    k = 1 / np.sqrt(H)
    w = dict(w_ih=rng.uniform(-k, k, (3 * H, I)), w_hh=rng.uniform(-k, k, (3 * H, H)),
             b_ih=rng.uniform(-k, k, 3 * H), b_hh=rng.uniform(-k, k, 3 * H))
    x = rng.standard_normal((B, T, I))
    h0 = rng.standard_normal((B, H))
    dout = rng.standard_normal((B, T, H))
    dhn = rng.standard_normal((B, H))
    f32 = lambda a: a.astype(np.float32)
    return {k2: f32(v) for k2, v in dict(x=x, h0=h0, dout=dout, dhn=dhn, **w).items()}


def _run_capi(B, T, I, H, with_dout, offset=0, seed=None):
    """Forward + backward through the C ABI vs the FP64 oracle.  With offset k
    every caller-owned buffer starts k floats into its allocation (k = 1:
    4-byte aligned only, so every 16-byte fast path must step aside)."""
    lib = _lib.load()
    c = _case(B, T, I, H, seed=B * 1000 + H if seed is None else seed)
    # Oracle in float64 on the float32-rounded inputs.
    d64 = {k: v.astype(np.float64) for k, v in c.items()}
    out_o, hn_o, st = O.gru_layer_forward(d64["x"], d64["h0"], d64["w_ih"], d64["w_hh"], d64["b_ih"], d64["b_hh"])
    g = O.gru_layer_backward(d64["dout"] if with_dout else None, d64["dhn"], d64["x"], d64["w_ih"], d64["w_hh"], st)

    dev = torch.device("cuda")

    def buf(*shape, like=None):
        n = int(np.prod(shape))
        base = torch.empty(n + offset, device=dev)
        v = base[offset:].view(*shape)
        if like is not None:
            v.copy_(torch.from_numpy(like))
        return v

    t = {k: buf(*v.shape, like=v) for k, v in c.items()}
    out = buf(B, T, H)
    hn = buf(B, H)
    stash = buf(lib.gru_stash_bytes(B, T, H) // 4)
    wsf = lib.gru_forward_workspace_bytes(B, T, I, H)
    ws = torch.empty(wsf, dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.gru_forward(_p(t["x"]), _p(t["h0"]), _p(t["w_ih"]), _p(t["w_hh"]), _p(t["b_ih"]), _p(t["b_hh"]),
                         _p(out), _p(hn), _p(stash), _p(ws), wsf, B, T, I, H, s)
    assert rc == 0, _lib.last_error()
    grads = {k: buf(*shape) for k, shape in dict(
        dx=(B, T, I), dh0=(B, H), dw_ih=(3 * H, I), dw_hh=(3 * H, H), db_ih=(3 * H,), db_hh=(3 * H,)).items()}
    wsb = lib.gru_backward_workspace_bytes(B, T, I, H)
    ws2 = torch.empty(wsb, dtype=torch.uint8, device=dev)
    rc = lib.gru_backward(_p(t["dout"]) if with_dout else None, _p(t["dhn"]), _p(t["x"]), _p(t["w_ih"]),
                          _p(t["w_hh"]), _p(stash), _p(grads["dx"]), _p(grads["dh0"]), _p(grads["dw_ih"]),
                          _p(grads["dw_hh"]), _p(grads["db_ih"]), _p(grads["db_hh"]), _p(ws2), wsb,
                          B, T, I, H, s)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), out_o, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(hn.cpu().numpy(), hn_o, rtol=RTOL, atol=ATOL)
    # The stash holds r, z, n, W_hn.h+b_hn and h_prev per (b, t).
    st_gpu = stash.view(B, T, 5, H).cpu().numpy()
    for i, k in enumerate(("r", "z", "n", "hn", "h_prev")):
        np.testing.assert_allclose(st_gpu[:, :, i], st[k], rtol=RTOL, atol=ATOL, err_msg=k)
    for k in grads:
        np.testing.assert_allclose(grads[k].cpu().numpy(), g[k], rtol=RTOL, atol=ATOL, err_msg=k)


@pytest.mark.parametrize("B,T,I,H", [(3, 7, 5, 33), (4, 16, 64, 256), (2, 5, 3, 129), (17, 4, 2, 20)])
@pytest.mark.parametrize("with_dout", [True, False])
def test_capi_forward_backward_vs_oracle(B, T, I, H, with_dout):
    _run_capi(B, T, I, H, with_dout)


@pytest.mark.parametrize("B,T,I,H", [(4, 9, 32, 64), (3, 6, 8, 256), (2, 5, 12, 128)])
def test_capi_unaligned_caller_buffers(B, T, I, H):
    # every caller pointer 4 bytes past a 16-byte boundary
    _run_capi(B, T, I, H, True, offset=1)


def test_capi_long_sequence():
    # many passes through the input ring and both mbarrier phases
    _run_capi(3, 2500, 16, 130, True, seed=2500)


def test_capi_inference_without_stash():
    lib = _lib.load()
    B, T, I, H = 5, 6, 7, 90
    c = _case(B, T, I, H, seed=11)
    d64 = {k: v.astype(np.float64) for k, v in c.items()}
    out_o, hn_o, _ = O.gru_layer_forward(d64["x"], d64["h0"], d64["w_ih"], d64["w_hh"], d64["b_ih"], d64["b_hh"])
    t = {k: torch.from_numpy(v).cuda() for k, v in c.items()}
    out = torch.empty(B, T, H, device="cuda")
    hn = torch.empty(B, H, device="cuda")
    wsf = lib.gru_forward_workspace_bytes(B, T, I, H)
    ws = torch.empty(wsf, dtype=torch.uint8, device="cuda")
    rc = lib.gru_forward(_p(t["x"]), _p(t["h0"]), _p(t["w_ih"]), _p(t["w_hh"]), _p(t["b_ih"]), _p(t["b_hh"]),
                         _p(out), _p(hn), None, _p(ws), wsf, B, T, I, H, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    np.testing.assert_allclose(out.cpu().numpy(), out_o, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(hn.cpu().numpy(), hn_o, rtol=RTOL, atol=ATOL)


def test_capi_error_codes():
    lib = _lib.load()
    B, T, I, H = 2, 3, 4, 8
    x = torch.zeros(B, T, I, device="cuda")
    h0 = torch.zeros(B, H, device="cuda")
    w = torch.zeros(3 * H, max(I, H), device="cuda")
    b = torch.zeros(3 * H, device="cuda")
    out = torch.empty(B, T, H, device="cuda")
    hn = torch.empty(B, H, device="cuda")
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.gru_forward(_p(x), _p(h0), _p(w), _p(w), _p(b), _p(b), _p(out), _p(hn), None, _p(ws), 16, B, T, I, H, s)
    assert rc == 1 and "workspace" in _lib.last_error()
    rc = lib.gru_forward(_p(x), _p(h0), _p(w), _p(w), _p(b), _p(b), _p(out), _p(hn), None, _p(ws), 16, B, T, I, 300, s)
    assert rc == 3 and "256" in _lib.last_error()
    rc = lib.gru_forward(None, _p(h0), _p(w), _p(w), _p(b), _p(b), _p(out), _p(hn), None, _p(ws), 16, B, T, I, H, s)
    assert rc == 1 and "null" in _lib.last_error()
    # A good call clears the error text.
    wsf = lib.gru_forward_workspace_bytes(B, T, I, H)
    ws = torch.empty(wsf, dtype=torch.uint8, device="cuda")
    rc = lib.gru_forward(_p(x), _p(h0), _p(w), _p(w), _p(b), _p(b), _p(out), _p(hn), None, _p(ws), wsf, B, T, I, H, s)
    assert rc == 0 and _lib.last_error() == ""
