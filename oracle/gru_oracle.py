"""NumPy restatement of the reference GRU forward/backward (test oracle).

This module is TEST INFRASTRUCTURE.  It is a CPU checker for the CUDA path in
``rnn_kernel_b200``; the product never imports it.

Parity is pinned: ``tests/golden/*.npz`` were produced by running the
reference's own pure-torch ``CustomGRU`` (plus torch autograd) and
``torch.nn.GRU`` at several small shapes, and ``tests/test_oracle.py`` checks
this restatement against every fixture.

Reference anchors (paths inside HanXuxx/RNN_kernel):

* forward math, gate order r,z,n and the ``F.linear`` + ``chunk(3)`` layout:
  ``src/rnn_kernel/custom_gru.py:76-122``;
* the forward stash ``{r, z, n, W_hn.h + b_hn}``:
  ``src/rnn_kernel/a100/prod/kernels/a100_gru_h256_kernels.cu:758-775``;
* the backward pointwise formulas and the split of ``dG_ih`` / ``dG_hh``:
  ``src/rnn_kernel/a100/prod/kernels/a100_gru_h256_kernels.cu:852-866``;
* the weight/input-gradient contractions and the ``grad_h_n`` plumbing:
  ``src/rnn_kernel/a100/prod/gru.py:532-580``.

Every function works in the dtype of its inputs (float32 or float64), so the
same code gives an FP32 restatement and an FP64 "truth".
"""
from __future__ import annotations

import numpy as np


def _sigmoid(v: np.ndarray) -> np.ndarray:
    one = v.dtype.type(1.0)
    return one / (one + np.exp(-v))


def gru_layer_forward(x, h0, w_ih, w_hh, b_ih, b_hh):
    """One GRU layer, batch_first.

    x [B,T,I], h0 [B,H], w_ih [3H,I], w_hh [3H,H], b_ih/b_hh [3H].
    Returns ``(out [B,T,H], h_n [B,H], stash)`` where ``stash`` is a dict of
    ``r, z, n, hn`` (each [B,T,H], ``hn = W_hn.h_prev + b_hn``) and
    ``h_prev`` [B,T,H] (the hidden state each step started from).

    Follows ``custom_gru.py:97-122``: input gates for all timesteps first, then
    the step loop ``r=sig(i_r+h_r); z=sig(i_z+h_z); n=tanh(i_n+r*h_n);
    h' = n + z*(h-n)``.
    """
    B, T, I = x.shape
    H = w_hh.shape[1]
    dt = x.dtype
    gi = (x.reshape(B * T, I) @ w_ih.T + b_ih).reshape(B, T, 3 * H)
    out = np.empty((B, T, H), dt)
    st = {k: np.empty((B, T, H), dt) for k in ("r", "z", "n", "hn", "h_prev")}
    h = h0.astype(dt, copy=True)
    for t in range(T):
        gh = h @ w_hh.T + b_hh
        i_r, i_z, i_n = gi[:, t, :H], gi[:, t, H:2 * H], gi[:, t, 2 * H:]
        h_r, h_z, h_n = gh[:, :H], gh[:, H:2 * H], gh[:, 2 * H:]
        r = _sigmoid(i_r + h_r)
        z = _sigmoid(i_z + h_z)
        n = np.tanh(i_n + r * h_n)
        st["h_prev"][:, t] = h
        h = n + z * (h - n)
        out[:, t] = h
        st["r"][:, t], st["z"][:, t], st["n"][:, t], st["hn"][:, t] = r, z, n, h_n
    return out, h.copy(), st


def gru_layer_backward(dout, dhn, x, w_ih, w_hh, stash):
    """Backward of :func:`gru_layer_forward`.

    dout [B,T,H] (may be None -> zeros), dhn [B,H] (may be None -> zeros).
    Returns dict with dx, dh0, dw_ih, dw_hh, db_ih, db_hh and the per-step
    gate gradients dG_ih / dG_hh ([B,T,3H]).

    Pointwise formulas follow ``a100_gru_h256_kernels.cu:852-866``::

        g      = dh_rec + dout[t]
        dz     = g*(h_prev-n);  dn = g*(1-z);  dn_pre = dn*(1-n^2)
        dr     = dn_pre*hn;     dhn_gate = dn_pre*r
        dr_pre = dr*r*(1-r);    dz_pre = dz*z*(1-z)
        dh_prev = g*z + dG_hh . W_hh
        dG_ih = [dr_pre, dz_pre, dn_pre];  dG_hh = [dr_pre, dz_pre, dhn_gate]

    and the contractions follow ``prod/gru.py:569-578``.
    """
    r, z, n, hn, hp = (stash[k] for k in ("r", "z", "n", "hn", "h_prev"))
    B, T, H = r.shape
    I = x.shape[2]
    dt = r.dtype
    one = dt.type(1.0)
    if dout is None:
        dout = np.zeros((B, T, H), dt)
    dh = np.zeros((B, H), dt) if dhn is None else dhn.astype(dt, copy=True)
    dgi = np.empty((B, T, 3 * H), dt)
    dgh = np.empty((B, T, 3 * H), dt)
    for t in range(T - 1, -1, -1):
        g = dh + dout[:, t]
        rt, zt, nt, hnt, hpt = r[:, t], z[:, t], n[:, t], hn[:, t], hp[:, t]
        dz = g * (hpt - nt)
        dn = g * (one - zt)
        dn_pre = dn * (one - nt * nt)
        dr = dn_pre * hnt
        dhn_gate = dn_pre * rt
        dr_pre = dr * rt * (one - rt)
        dz_pre = dz * zt * (one - zt)
        dgi[:, t] = np.concatenate([dr_pre, dz_pre, dn_pre], axis=1)
        dgh[:, t] = np.concatenate([dr_pre, dz_pre, dhn_gate], axis=1)
        dh = g * zt + dgh[:, t] @ w_hh
    dgi2 = dgi.reshape(B * T, 3 * H)
    dgh2 = dgh.reshape(B * T, 3 * H)
    return {
        "dx": (dgi2 @ w_ih).reshape(B, T, I),
        "dh0": dh,
        "dw_ih": dgi2.T @ x.reshape(B * T, I),
        "dw_hh": dgh2.T @ hp.reshape(B * T, H),
        "db_ih": dgi2.sum(axis=0),
        "db_hh": dgh2.sum(axis=0),
        "dG_ih": dgi,
        "dG_hh": dgh,
    }


def gru_forward(x, hx, params):
    """Stacked GRU forward. ``params`` is a list of (w_ih, w_hh, b_ih, b_hh)
    per layer, ``hx`` is [L,B,H].  Returns (out, h_n [L,B,H], stashes)."""
    layer_in = x
    hns, stashes, inputs = [], [], []
    for l, (w_ih, w_hh, b_ih, b_hh) in enumerate(params):
        inputs.append(layer_in)
        layer_in, hn, st = gru_layer_forward(layer_in, hx[l], w_ih, w_hh, b_ih, b_hh)
        hns.append(hn)
        stashes.append(st)
    return layer_in, np.stack(hns), (stashes, inputs)


def gru_backward(dout, dhn, params, saved):
    """Stacked GRU backward.  ``dhn`` [L,B,H] (or None).  Returns
    (dx, dh0 [L,B,H], [per-layer dict of dw_ih, dw_hh, db_ih, db_hh])."""
    stashes, inputs = saved
    L = len(params)
    grads = [None] * L
    dh0 = [None] * L
    g = dout
    for l in range(L - 1, -1, -1):
        w_ih, w_hh, _, _ = params[l]
        res = gru_layer_backward(g, None if dhn is None else dhn[l], inputs[l], w_ih, w_hh, stashes[l])
        grads[l] = {k: res[k] for k in ("dw_ih", "dw_hh", "db_ih", "db_hh")}
        dh0[l] = res["dh0"]
        g = res["dx"]
    return g, np.stack(dh0), grads
