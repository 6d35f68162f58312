"""Time chunks: the forward and backward run as n consecutive chunks of the
sequence, with one chunk's tensor-core products on a side stream beside the
loop over another.  Checked through the C ABI against the FP64 oracle for
every chunk count, and against the unchunked run: the forward (outputs, h_n,
stash) and every gradient but the weight gradients are bit-identical; the
weight gradients differ only in how their split-K partial sums are grouped."""
import numpy as np
import pytest
import torch

from oracle import gru_oracle as O
from rnn_kernel_b200 import _lib
from tests.test_capi_gpu import _case, _p, _run_capi

pytestmark = pytest.mark.gpu


@pytest.fixture
def chunks():
    prev = _lib.set_time_chunks(0)
    yield _lib.set_time_chunks
    _lib.set_time_chunks(prev)


@pytest.mark.parametrize("B,T,I,H,n", [(4, 256, 16, 64, 2), (3, 512, 24, 256, 2), (3, 512, 24, 256, 4),
                                       (5, 384, 8, 129, 3), (2, 256, 5, 33, 2)])
@pytest.mark.parametrize("with_dout", [True, False])
def test_chunked_vs_oracle(chunks, B, T, I, H, n, with_dout):
    chunks(n)
    _run_capi(B, T, I, H, with_dout, seed=31 * T + H)


def _fwd_bwd(B, T, I, H, seed):
    lib = _lib.load()
    c = _case(B, T, I, H, seed)
    t = {k: torch.from_numpy(v).cuda() for k, v in c.items()}
    out = torch.empty(B, T, H, device="cuda")
    hn = torch.empty(B, H, device="cuda")
    stash = torch.empty(lib.gru_stash_bytes(B, T, H) // 4, device="cuda")
    wsf = lib.gru_forward_workspace_bytes(B, T, I, H)
    ws = torch.empty(wsf, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.gru_forward(_p(t["x"]), _p(t["h0"]), _p(t["w_ih"]), _p(t["w_hh"]), _p(t["b_ih"]), _p(t["b_hh"]),
                         _p(out), _p(hn), _p(stash), _p(ws), wsf, B, T, I, H, s)
    assert rc == 0, _lib.last_error()
    g = {k: torch.empty(*shape, device="cuda") for k, shape in dict(
        dx=(B, T, I), dh0=(B, H), dw_ih=(3 * H, I), dw_hh=(3 * H, H), db_ih=(3 * H,), db_hh=(3 * H,)).items()}
    wsb = lib.gru_backward_workspace_bytes(B, T, I, H)
    ws2 = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    rc = lib.gru_backward(_p(t["dout"]), _p(t["dhn"]), _p(t["x"]), _p(t["w_ih"]), _p(t["w_hh"]), _p(stash),
                          _p(g["dx"]), _p(g["dh0"]), _p(g["dw_ih"]), _p(g["dw_hh"]), _p(g["db_ih"]), _p(g["db_hh"]),
                          _p(ws2), wsb, B, T, I, H, s)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return dict(out=out, hn=hn, stash=stash, **g)


@pytest.mark.parametrize("B,T,I,H", [(64, 512, 256, 256), (16, 256, 96, 96)])
def test_chunked_matches_unchunked(chunks, B, T, I, H):
    chunks(1)
    ref = _fwd_bwd(B, T, I, H, seed=7)
    c = {k: v.astype(np.float64) for k, v in _case(B, T, I, H, 7).items()}
    _, _, st = O.gru_layer_forward(c["x"], c["h0"], c["w_ih"], c["w_hh"], c["b_ih"], c["b_hh"])
    truth = O.gru_layer_backward(c["dout"], c["dhn"], c["x"], c["w_ih"], c["w_hh"], st)
    for n in (2, 4):
        if T % (128 * n):
            continue
        chunks(n)
        got = _fwd_bwd(B, T, I, H, seed=7)
        for k in ("out", "hn", "stash", "dx", "dh0"):
            assert torch.equal(got[k], ref[k]), (n, k)
        for k in ("db_ih", "db_hh"):
            # FP64 per-chunk sums: only the grouping of the FP64 additions differs
            torch.testing.assert_close(got[k], ref[k], rtol=1e-6, atol=1e-7)
        for k in ("dw_ih", "dw_hh"):
            # The same products with the K = B*T sum split differently (unit-
            # scale upstream gradients: sums of 3e4 terms of size ~1, where
            # even torch FP32 misses the element-wise bar, so normwise): close
            # to the FP64 truth, and chunking does not make the max error
            # larger than 1.25x the unchunked one.
            t = truth[k]
            a = got[k].double().cpu().numpy()
            e_got = np.abs(a - t).max()
            e_ref = np.abs(ref[k].double().cpu().numpy() - t).max()
            rel = np.linalg.norm(a - t) / np.linalg.norm(t)
            print(f"{k} chunks={n}: max error {e_got:.3e} (unchunked {e_ref:.3e}), normwise {rel:.1e}")
            assert rel < 1e-6, (n, k, rel)
            assert e_got <= 1.25 * e_ref + 1e-7, (n, k, e_got, e_ref)


def test_knob_rejects_bad_values():
    assert _lib.load().gru_set_time_chunks(5) == -1
    assert _lib.load().gru_set_time_chunks(-1) == -1
