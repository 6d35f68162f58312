"""Host-side API checks that need no GPU (mirrors tests/test_a100_prod.py:19-81
of the reference: rejection rules, CPU-safe availability probe, import
isolation) plus the C-ABI library export check."""
import ctypes
import json
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from rnn_kernel_b200 import GRU, from_torch_gru, is_b200_available, is_supported_gru
from rnn_kernel_b200 import _lib, build

ROOT = Path(__file__).resolve().parent.parent


def test_rejects_unsupported_torch_gru():
    assert is_supported_gru(torch.nn.GRU(5, 128, batch_first=True))
    assert is_supported_gru(torch.nn.GRU(300, 256, num_layers=6, batch_first=True))
    assert not is_supported_gru(torch.nn.GRU(5, 257, batch_first=True))
    assert not is_supported_gru(torch.nn.GRU(5, 64, batch_first=False))
    assert not is_supported_gru(torch.nn.GRU(5, 64, batch_first=True, bidirectional=True))
    assert not is_supported_gru(torch.nn.GRU(5, 64, num_layers=2, dropout=0.1, batch_first=True))
    assert not is_supported_gru(torch.nn.GRU(5, 64, batch_first=True, bias=False))
    assert not is_supported_gru(torch.nn.GRU(5, 64, batch_first=True).double())
    assert not is_supported_gru(torch.nn.LSTM(5, 64, batch_first=True))
    with pytest.raises(ValueError, match="hidden_size"):
        GRU(input_size=5, hidden_size=257)
    with pytest.raises(ValueError, match="hidden_size"):
        GRU(input_size=5, hidden_size=0)
    with pytest.raises(ValueError, match="num_layers"):
        GRU(input_size=5, num_layers=0)
    with pytest.raises(ValueError, match="input_size"):
        GRU(input_size=0)
    with pytest.raises(ValueError, match="batch_first"):
        GRU(input_size=4, batch_first=False)
    with pytest.raises(ValueError, match="bias"):
        GRU(input_size=4, bias=False)
    with pytest.raises(ValueError, match="dropout"):
        GRU(input_size=4, num_layers=2, dropout=0.5)
    with pytest.raises(ValueError, match="hidden_size <= 256"):
        from_torch_gru(torch.nn.GRU(5, 300, batch_first=True))


def test_module_matches_nn_gru_layout_and_init():
    torch.manual_seed(0)
    g = GRU(7, 33, num_layers=3)
    ref = torch.nn.GRU(7, 33, num_layers=3, batch_first=True)
    assert [n for n, _ in g.named_parameters()] == [n for n, _ in ref.named_parameters()]
    for (n, p), (_, q) in zip(g.named_parameters(), ref.named_parameters()):
        assert p.shape == q.shape, n
        assert p.abs().max() <= 1 / 33 ** 0.5 + 1e-7
    g.load_state_dict(ref.state_dict())
    m = from_torch_gru(ref)
    for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
        assert torch.equal(p, q), n


def test_is_b200_available_accepts_cpu_device():
    assert not is_b200_available(torch.device("cpu"))


def test_cpu_tensors_raise_runtime_error():
    g = GRU(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        g(torch.randn(2, 3, 4))
    with pytest.raises(ValueError, match="hx must have shape"):
        g(torch.randn(2, 3, 4), torch.zeros(2, 2, 8))


def test_import_does_not_load_cuda_library_or_compilers():
    script = """
import json, sys
import rnn_kernel_b200
from rnn_kernel_b200 import GRU, from_torch_gru
print(json.dumps({
    "lib_loaded": rnn_kernel_b200._lib._lib is not None,
    "nvrtc": "cuda.nvrtc" in sys.modules,
    "triton": "triton" in sys.modules,
    "oracle": any(m == "oracle" or m.startswith("oracle.") for m in sys.modules),
}))
"""
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", script], check=True, env=env, text=True, capture_output=True)
    assert json.loads(r.stdout.strip().splitlines()[-1]) == {
        "lib_loaded": False, "nvrtc": False, "triton": False, "oracle": False}


def _header_symbols():
    text = (ROOT / "include" / "rnn_kernel_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gru_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_header_symbol():
    lib = _lib.load()
    syms = _header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_size_queries_without_gpu():
    lib = _lib.load()
    assert lib.gru_stash_bytes(64, 512, 256) == 4 * 64 * 512 * 5 * 256
    assert lib.gru_forward_workspace_bytes(64, 512, 256, 256) >= 4 * 64 * 512 * 768
    assert lib.gru_backward_workspace_bytes(64, 512, 256, 256) >= 2 * 4 * 64 * 512 * 768
    assert lib.gru_stash_bytes(0, 5, 4) == 0
    assert lib.gru_device_supported(0) in (0, 1)
    assert lib.gru_device_supported(-1) == 0


def test_library_built_for_sm100a():
    # The in-tree library is built by nvcc for sm_100a only; check the build flags.
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)
    assert build.LIB_PATH.exists()
