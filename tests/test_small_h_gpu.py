"""Time loops for small hidden sizes: the single-CTA kernels (one CTA per
group of 1, 2 or 4 batch rows, W_hh in registers, one barrier per step; the
forward for H <= 96, the backward for H <= 64), checked through the C ABI
against the FP64 oracle and against the thread-block-cluster kernels
(gru_set_small_loops(1)) on the same inputs.

Cases cover both K-slice widths (H <= 64 and 64 < H <= 96), 1, 2 and 4 rows
per CTA (B above one and two CTAs per SM), the bulk-copy path (H % 4 == 0,
16-byte-aligned buffers) and the per-lane path (odd H, or buffers offset by
one float), with and without an output gradient."""
import pytest
import torch

from rnn_kernel_b200 import _lib
from tests.test_capi_gpu import _run_capi
from tests.test_time_chunks_gpu import _fwd_bwd

pytestmark = pytest.mark.gpu


@pytest.fixture
def small_mode():
    prev = _lib.set_small_loops(0)
    yield _lib.set_small_loops
    _lib.set_small_loops(prev)


@pytest.mark.parametrize("B,T,I,H,offset", [
    (1, 40, 5, 8, 0),        # one warp, bulk rows of 32 bytes
    (3, 33, 7, 33, 0),       # odd H: per-lane copies
    (64, 48, 64, 64, 0),     # the sweep's shape class, bulk
    (64, 48, 64, 64, 1),     # same, buffers 4-byte aligned only: per-lane copies
    (200, 24, 16, 64, 0),    # 2 rows per CTA
    (300, 16, 8, 96, 0),     # 4 rows per CTA, 24-column K slices
    (150, 20, 12, 65, 0),    # 2 rows per CTA, odd H, 24-column K slices
    (5, 30, 3, 96, 0),
])
@pytest.mark.parametrize("with_dout", [True, False])
def test_small_h_vs_oracle(small_mode, B, T, I, H, offset, with_dout):
    small_mode(0)
    _run_capi(B, T, I, H, with_dout, offset=offset, seed=7 * B + H)


@pytest.mark.parametrize("B,T,I,H", [(64, 128, 32, 64), (7, 64, 16, 96), (9, 50, 4, 31), (200, 40, 8, 32)])
def test_small_h_matches_cluster_kernels(small_mode, B, T, I, H):
    small_mode(0)
    a = _fwd_bwd(B, T, I, H, seed=H)
    small_mode(1)
    b = _fwd_bwd(B, T, I, H, seed=H)
    small_mode(0)
    for k in a:
        torch.testing.assert_close(a[k], b[k], rtol=1e-4, atol=1e-5, msg=lambda m, k=k: f"{k}: {m}")


def test_small_loops_knob_rejects_bad_mode():
    assert _lib.load().gru_set_small_loops(2) == -1
    assert _lib.load().gru_set_small_loops(-1) == -1
