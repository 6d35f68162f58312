"""gru_forward_inference_noalloc through the C ABI.

This entry point is for callers that cannot allocate device memory (a plugin
whose host owns all device memory through its own allocator, or code running
where an allocation is not allowed): it takes no workspace and uses a static
device array inside the library instead.  Its results must equal the regular
gru_forward(stash = NULL) with a caller workspace, call after call, because
every call reuses the same array.  This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from rnn_kernel_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5
MAX_BYTES = 16 << 20


def _p(t):
    return None if t is None else t.data_ptr()


def _inputs(B, T, I, H, seed):
    g = torch.Generator().manual_seed(seed)
    k = 1.0 / H ** 0.5
    u = lambda *s: ((torch.rand(*s, generator=g) * 2 - 1) * k).cuda()
    return dict(x=torch.randn(B, T, I, generator=g).cuda(), h0=torch.randn(B, H, generator=g).cuda(),
                w_ih=u(3 * H, I), w_hh=u(3 * H, H), b_ih=u(3 * H), b_hh=u(3 * H))


def _regular(lib, c, B, T, I, H):
    out = torch.empty(B, T, H, device="cuda")
    hn = torch.empty(B, H, device="cuda")
    n = lib.gru_forward_workspace_bytes(B, T, I, H)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
    rc = lib.gru_forward(_p(c["x"]), _p(c["h0"]), _p(c["w_ih"]), _p(c["w_hh"]), _p(c["b_ih"]), _p(c["b_hh"]),
                         _p(out), _p(hn), None, _p(ws), n, B, T, I, H, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return out, hn


def _noalloc(lib, c, B, T, I, H):
    out = torch.empty(B, T, H, device="cuda")
    hn = torch.empty(B, H, device="cuda")
    rc = lib.gru_forward_inference_noalloc(_p(c["x"]), _p(c["h0"]), _p(c["w_ih"]), _p(c["w_hh"]), _p(c["b_ih"]),
                                           _p(c["b_hh"]), _p(out), _p(hn), B, T, I, H,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return out, hn


@pytest.mark.parametrize("shape", [(8, 64, 256, 256), (3, 9, 5, 130)])
def test_noalloc_matches_regular_forward_twice(shape):
    B, T, I, H = shape
    lib = _lib.load()
    # Two calls in a row with different inputs: the second must not see the
    # first call's leftovers in the shared static scratch.
    for seed in (1, 2):
        c = _inputs(B, T, I, H, seed)
        ref_out, ref_hn = _regular(lib, c, B, T, I, H)
        out, hn = _noalloc(lib, c, B, T, I, H)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref_out.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(hn.cpu().numpy(), ref_hn.cpu().numpy(), rtol=RTOL, atol=ATOL)
    assert _lib.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    B, T, I, H = 64, 512, 256, 256  # needs 96 MiB of input gates
    assert lib.gru_forward_workspace_bytes(B, T, I, H) > MAX_BYTES
    c = {k: torch.zeros(1, device="cuda") for k in ("x", "h0", "w_ih", "w_hh", "b_ih", "b_hh")}
    out = torch.zeros(1, device="cuda")
    rc = lib.gru_forward_inference_noalloc(_p(c["x"]), _p(c["h0"]), _p(c["w_ih"]), _p(c["w_hh"]), _p(c["b_ih"]),
                                           _p(c["b_hh"]), _p(out), _p(out), B, T, I, H,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.GRU_ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
