"""``torch.nn.GRU``-compatible FP32 GRU on B200, backed by the C-ABI CUDA library.

Mirrors the reference's prod surface (``src/rnn_kernel/a100/prod/gru.py``):

* :class:`GRUFunction` — ``apply(x, h0, W_ih, W_hh, b_ih, b_hh) ->
  (output [B,T,H], h_n [1,B,H])`` with backward returning ``(dx, dh0, dW_ih,
  dW_hh, db_ih, db_hh)`` (ref ``_A100GRUFunction``, ``:488-580``);
* :class:`GRU` — the ``nn.Module`` (ref ``A100GRU``, ``:620-786``) with
  ``forward(x, hx=None) -> (output, h_n [L,B,H])``, ``forward_inference``,
  ``forward_output_only`` and
  the automatic no-stash path under ``torch.no_grad()`` (``:761-778``);
* :func:`from_torch_gru`, :func:`is_supported_gru`, :func:`is_b200_available`
  (ref ``from_torch_gru`` ``:789-808``, ``is_supported_gru`` ``:120-136``,
  ``is_a100_available`` ``:109-117``).

Validation follows ``_validate_inputs`` (``:184-223``): shape problems raise
``ValueError``, device/dtype problems raise ``RuntimeError``, and CUDA
failures raise ``RuntimeError`` with the library's message.  There is no CPU
fallback: use :func:`is_supported_gru` to decide between this module and
``torch.nn.GRU``.

Supported range (wider than the reference's H=256, I<=16, L<=4): any
``1 <= hidden_size <= 256``, any ``input_size >= 1``, any number of layers,
batch_first, unidirectional, bias, no dropout, float32.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from . import _lib

MAX_HIDDEN_SIZE = 256


def _device_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError("device must be a CUDA device.")
    return torch.cuda.current_device() if d.index is None else d.index


def is_b200_available(device=None) -> bool:
    """True when ``device`` (default: current) is a compute-capability 10.x GPU."""
    if not torch.cuda.is_available():
        return False
    try:
        idx = _device_index(device)
    except ValueError:
        return False
    return torch.cuda.get_device_capability(idx)[0] == 10


def is_supported_gru(gru: nn.Module) -> bool:
    """Whether ``gru`` (a ``torch.nn.GRU``) can be replaced by :class:`GRU` losslessly."""
    if not isinstance(gru, nn.GRU) or not gru.bias:
        return False
    try:
        p = next(gru.parameters())
    except StopIteration:
        return False
    return (
        gru.input_size >= 1
        and 1 <= gru.hidden_size <= MAX_HIDDEN_SIZE
        and gru.num_layers >= 1
        and gru.batch_first
        and not gru.bidirectional
        and gru.dropout == 0.0
        and p.dtype == torch.float32
    )


def _validate(x, h0, w_ih, w_hh, b_ih, b_hh):
    if not x.is_cuda:
        raise RuntimeError("rnn_kernel_b200 GRU requires CUDA tensors.")
    if x.dim() != 3:
        raise ValueError("x must have shape [batch, seq, input].")
    if h0.dim() != 2:
        raise ValueError("h0 must have shape [batch, hidden].")
    H = h0.size(1)
    if not 1 <= H <= MAX_HIDDEN_SIZE:
        raise ValueError(f"hidden_size must be in [1, {MAX_HIDDEN_SIZE}].")
    tensors = (x, h0, w_ih, w_hh, b_ih, b_hh)
    if len({t.device for t in tensors}) != 1:
        raise ValueError("All tensors must be on the same CUDA device.")
    if any(t.dtype != torch.float32 for t in tensors):
        raise RuntimeError("rnn_kernel_b200 GRU supports float32 only.")
    B, T, I = x.shape
    if h0.size(0) != B:
        raise ValueError("h0 batch dimension must match x.")
    if I < 1:
        raise ValueError("input_size must be >= 1.")
    if tuple(w_ih.shape) != (3 * H, I):
        raise ValueError("weight_ih must have shape [3 * hidden, input].")
    if tuple(w_hh.shape) != (3 * H, H):
        raise ValueError("weight_hh must have shape [3 * hidden, hidden].")
    if tuple(b_ih.shape) != (3 * H,) or tuple(b_hh.shape) != (3 * H,):
        raise ValueError("bias tensors must have shape [3 * hidden].")
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    if not is_b200_available(dev):
        raise RuntimeError("rnn_kernel_b200 requires a B200-class (sm_100) GPU.")
    return B, T, I, H, dev


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _forward_impl(x, h0, w_ih, w_hh, b_ih, b_hh, train: bool):
    B, T, I, H, dev = _validate(x, h0, w_ih, w_hh, b_ih, b_hh)
    lib = _lib.load()
    with torch.cuda.device(dev):
        x, h0, w_ih, w_hh, b_ih, b_hh = (t.contiguous() for t in (x, h0, w_ih, w_hh, b_ih, b_hh))
        out = torch.empty(B, T, H, device=x.device, dtype=torch.float32)
        hn = torch.empty(1, B, H, device=x.device, dtype=torch.float32)
        stash = None
        if train and B * T > 0:
            stash = torch.empty(lib.gru_stash_bytes(B, T, H) // 4, device=x.device, dtype=torch.float32)
        ws_bytes = lib.gru_forward_workspace_bytes(B, T, I, H)
        ws = torch.empty(max(ws_bytes, 1), device=x.device, dtype=torch.uint8)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(
            lib.gru_forward(_ptr(x), _ptr(h0), _ptr(w_ih), _ptr(w_hh), _ptr(b_ih), _ptr(b_hh),
                            _ptr(out), _ptr(hn), _ptr(stash), _ptr(ws), ws_bytes, B, T, I, H, stream),
            "gru_forward",
        )
    return out, hn, stash, (x, w_ih, w_hh)


class GRUFunction(torch.autograd.Function):
    """One GRU layer: ``(x, h0, W_ih, W_hh, b_ih, b_hh) -> (output, h_n[1,B,H])``."""

    @staticmethod
    def forward(ctx, x, h0, weight_ih, weight_hh, bias_ih, bias_hh):
        out, hn, stash, (xc, w_ih, w_hh) = _forward_impl(x, h0, weight_ih, weight_hh, bias_ih, bias_hh, True)
        # an output the loss does not use arrives as None (the C ABI takes NULL
        # for it) instead of a materialised zero tensor
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(xc, w_ih, w_hh, stash if stash is not None else out.new_empty(0))
        ctx.shape = (x.size(0), x.size(1), x.size(2), h0.size(1))
        return out, hn

    @staticmethod
    def backward(ctx, grad_output, grad_h_n):
        x, w_ih, w_hh, stash = ctx.saved_tensors
        B, T, I, H = ctx.shape
        dev = x.device
        lib = _lib.load()
        with torch.cuda.device(dev):
            dout = None if grad_output is None else grad_output.contiguous()
            dhn = None if grad_h_n is None else grad_h_n.reshape(B, H).contiguous()
            dx = torch.empty(B, T, I, device=dev, dtype=torch.float32) if ctx.needs_input_grad[0] else None
            dh0 = torch.empty(B, H, device=dev, dtype=torch.float32)
            dw_ih = torch.empty(3 * H, I, device=dev, dtype=torch.float32)
            dw_hh = torch.empty(3 * H, H, device=dev, dtype=torch.float32)
            db_ih = torch.empty(3 * H, device=dev, dtype=torch.float32)
            db_hh = torch.empty(3 * H, device=dev, dtype=torch.float32)
            ws_bytes = lib.gru_backward_workspace_bytes(B, T, I, H)
            ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
            stream = torch.cuda.current_stream(dev).cuda_stream
            _lib.check(
                lib.gru_backward(_ptr(dout), _ptr(dhn), _ptr(x), _ptr(w_ih), _ptr(w_hh),
                                 _ptr(stash) if stash.numel() else None, _ptr(dx), _ptr(dh0),
                                 _ptr(dw_ih), _ptr(dw_hh), _ptr(db_ih), _ptr(db_hh),
                                 _ptr(ws), ws_bytes, B, T, I, H, stream),
                "gru_backward",
            )
        return dx, dh0, dw_ih, dw_hh, db_ih, db_hh


def gru_forward_inference(x, h0, weight_ih, weight_hh, bias_ih, bias_hh):
    """No-stash forward of one layer (ref ``_a100_gru_forward_inference``, ``:583-617``)."""
    with torch.no_grad():
        out, hn, _, _ = _forward_impl(x, h0, weight_ih, weight_hh, bias_ih, bias_hh, False)
    return out, hn


class GRU(nn.Module):
    """Drop-in ``torch.nn.GRU`` (batch_first) running the B200 kernels.

    Parameters are named ``weight_ih_l{k}``, ``weight_hh_l{k}``, ``bias_ih_l{k}``,
    ``bias_hh_l{k}`` with ``nn.GRU``'s shapes, so state dicts are
    interchangeable.
    """

    def __init__(self, input_size: int, hidden_size: int = 256, num_layers: int = 1,
                 batch_first: bool = True, bias: bool = True, dropout: float = 0.0) -> None:
        super().__init__()
        if not 1 <= hidden_size <= MAX_HIDDEN_SIZE:
            raise ValueError(f"GRU only supports 1 <= hidden_size <= {MAX_HIDDEN_SIZE}.")
        if input_size < 1:
            raise ValueError("GRU only supports input_size >= 1.")
        if num_layers < 1:
            raise ValueError("GRU only supports num_layers >= 1.")
        if not batch_first:
            raise ValueError("GRU only supports batch_first=True.")
        if not bias:
            raise ValueError("GRU currently requires bias=True.")
        if dropout != 0.0:
            raise ValueError("GRU currently requires dropout=0.")
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.num_layers = num_layers
        self.batch_first = batch_first
        self.bias = bias
        self.dropout = float(dropout)
        for layer in range(num_layers):
            li = input_size if layer == 0 else hidden_size
            setattr(self, f"weight_ih_l{layer}", nn.Parameter(torch.empty(3 * hidden_size, li)))
            setattr(self, f"weight_hh_l{layer}", nn.Parameter(torch.empty(3 * hidden_size, hidden_size)))
            setattr(self, f"bias_ih_l{layer}", nn.Parameter(torch.empty(3 * hidden_size)))
            setattr(self, f"bias_hh_l{layer}", nn.Parameter(torch.empty(3 * hidden_size)))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        stdv = 1.0 / math.sqrt(self.hidden_size)
        for w in self.parameters():
            nn.init.uniform_(w, -stdv, stdv)

    def layer_parameters(self, layer: int):
        return (getattr(self, f"weight_ih_l{layer}"), getattr(self, f"weight_hh_l{layer}"),
                getattr(self, f"bias_ih_l{layer}"), getattr(self, f"bias_hh_l{layer}"))

    def _prepare_hx(self, x: torch.Tensor, hx: Optional[torch.Tensor]) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError("x must have shape [batch, seq, input].")
        if hx is None:
            return x.new_zeros(self.num_layers, x.size(0), self.hidden_size)
        expected = (self.num_layers, x.size(0), self.hidden_size)
        if tuple(hx.shape) != expected:
            raise ValueError(f"hx must have shape {expected}.")
        return hx

    def _run(self, x, hx, train: bool):
        layer_in = x
        hns = []
        for layer in range(self.num_layers):
            params = self.layer_parameters(layer)
            if train:
                layer_in, hn = GRUFunction.apply(layer_in, hx[layer], *params)
            else:
                layer_in, hn = gru_forward_inference(layer_in, hx[layer], *params)
            hns.append(hn)
        return layer_in, (hns[0] if len(hns) == 1 else torch.cat(hns, dim=0))

    def forward(self, x: torch.Tensor, hx: Optional[torch.Tensor] = None):
        hx = self._prepare_hx(x, hx)
        if not torch.is_grad_enabled():
            return self._run(x, hx, train=False)
        return self._run(x, hx, train=True)

    def forward_inference(self, x: torch.Tensor, hx: Optional[torch.Tensor] = None):
        """Explicit forward-only, no-stash path."""
        hx = self._prepare_hx(x, hx)
        return self._run(x, hx, train=False)

    def forward_output_only(self, x: torch.Tensor, hx: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``output`` only, for callers that never use ``h_n`` (the reference
        harness's ``use_a100_output_only`` path, ``rnn_benchmark.py:521-522``;
        ref ``A100GRUH256.forward_output_only``, ``gru_autograd.py:5768-5777``).
        Trains through autograd when grad is enabled, else takes the no-stash
        path."""
        return self.forward(x, hx)[0]

    @classmethod
    def from_torch_gru(cls, gru: nn.GRU) -> "GRU":
        return from_torch_gru(gru)


def from_torch_gru(gru: nn.GRU) -> GRU:
    """Build a :class:`GRU` with the same weights as a supported ``torch.nn.GRU``."""
    if not is_supported_gru(gru):
        raise ValueError(
            "Only unidirectional batch_first float32 GRU with 1 <= hidden_size <= 256, "
            "bias=True and dropout=0 is supported."
        )
    device = next(gru.parameters()).device
    m = GRU(gru.input_size, gru.hidden_size, gru.num_layers, dropout=gru.dropout).to(device=device)
    with torch.no_grad():
        for layer in range(gru.num_layers):
            for name in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
                getattr(m, f"{name}_l{layer}").copy_(getattr(gru, f"{name}_l{layer}"))
    return m
