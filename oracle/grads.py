"""numpy restatement of the training backward of the two recurrences (test oracle).

Test infrastructure only: the GPU backward kernels are checked against these
functions, and these functions are checked against gradients that torch
autograd computes through the reference's own CPU recurrences
(tests/golden/grads_cases.npz, written by tests/golden/make_golden.py).

Both are written as explicit reverse-mode passes over the forward formulas,
in float64, saving every forward state (small cases only).

WKV-7 forward per token (``RWKV7TimeMix._torch_recurrence``,
yufmusicgen/model.py:156-164), state S [N, N], row i = value, column j = key::

    ret = exp(W_SCALE * sigmoid(w_raw)),  sa = S a,
    S' = S diag(ret) + sa b^T + v k^T,     y = S' r.

ROSA forward per token (``ROSAMemory._reference_recurrence``,
yufmusicgen/model.py:280-287, ungated read of the CUDA op,
rosa_householder.cu:89-91)::

    h = m - 2 (d.m) d,  m' = decay * h + sigmoid(write) * tanh(cand),
    read = m' - 2 (d.m') d.
"""

from __future__ import annotations

import numpy as np

W_SCALE = -0.6065306597  # yufmusicgen/model.py:156


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def wkv7_backward(r, w_raw, k, v, a, b, dy):
    """Gradients of sum(y * dy) for a zero initial state (the reference op has
    none, rwkv7_clampw.cu:25-29); the final state carries no gradient.

    All inputs [B, T, H, N]; returns (dr, dw_raw, dk, dv, da, db) float32.
    """
    r, w_raw, k, v, a, b, dy = (np.asarray(x, np.float64) for x in (r, w_raw, k, v, a, b, dy))
    B, T, H, N = r.shape
    sig = _sig(w_raw)
    ret = np.exp(W_SCALE * sig)
    # forward, keeping S_t (after token t) and sa_t
    S = np.zeros((B, H, N, N))
    states = np.empty((T + 1, B, H, N, N))
    states[0] = S
    sa = np.empty((B, T, H, N))
    for t in range(T):
        sa[:, t] = np.einsum("bhij,bhj->bhi", S, a[:, t])
        S = (S * ret[:, t][:, :, None, :] + sa[:, t][..., None] * b[:, t][:, :, None, :]
             + v[:, t][..., None] * k[:, t][:, :, None, :])
        states[t + 1] = S
    grads = {x: np.empty((B, T, H, N)) for x in ("r", "w", "k", "v", "a", "b")}
    G = np.zeros((B, H, N, N))  # dL/dS after token t
    for t in range(T - 1, -1, -1):
        S_new, S_old = states[t + 1], states[t]
        G = G + dy[:, t][..., None] * r[:, t][:, :, None, :]                   # y = S' r
        grads["r"][:, t] = np.einsum("bhij,bhi->bhj", S_new, dy[:, t])
        grads["v"][:, t] = np.einsum("bhij,bhj->bhi", G, k[:, t])
        grads["k"][:, t] = np.einsum("bhij,bhi->bhj", G, v[:, t])
        grads["b"][:, t] = np.einsum("bhij,bhi->bhj", G, sa[:, t])
        dsa = np.einsum("bhij,bhj->bhi", G, b[:, t])
        dret = np.einsum("bhij,bhij->bhj", G, S_old)
        grads["w"][:, t] = dret * ret[:, t] * W_SCALE * sig[:, t] * (1.0 - sig[:, t])
        grads["a"][:, t] = np.einsum("bhij,bhi->bhj", S_old, dsa)
        G = G * ret[:, t][:, :, None, :] + dsa[..., None] * a[:, t][:, :, None, :]
    return tuple(grads[x].astype(np.float32) for x in ("r", "w", "k", "v", "a", "b"))


def rosa_backward(cand, write, decay, direction, m0, dq):
    """Gradients of sum(read * dq) through the ungated ROSA scan.

    cand, write, dq [B, T, R] (pre-activation cand/write), decay [R]
    (post-sigmoid), direction [R] (used as given), m0 [B, R].  The read gate
    does not enter the ungated read, so its gradient is zero; the final memory
    carries no gradient.  Returns (d_cand, d_write, d_decay [B, T, R] per step,
    d_direction [B, R] per sequence, d_m0 [B, R]) float32.
    """
    cand, write, dq, m0 = (np.asarray(x, np.float64) for x in (cand, write, dq, m0))
    decay = np.asarray(decay, np.float64)
    d = np.asarray(direction, np.float64)
    B, T, R = cand.shape
    c = np.tanh(cand)
    wg = _sig(write)
    mem = np.empty((T + 1, B, R))
    mem[0] = m0
    for t in range(T):
        m = mem[t]
        h = m - 2.0 * (m @ d)[:, None] * d
        mem[t + 1] = decay * h + wg[:, t] * c[:, t]
    d_cand = np.empty((B, T, R))
    d_write = np.empty((B, T, R))
    d_decay = np.empty((B, T, R))
    d_dir = np.zeros((B, R))
    P = np.zeros((B, R))  # dL/dm_{t+1}
    for t in range(T - 1, -1, -1):
        m_old, m_new, q = mem[t], mem[t + 1], dq[:, t]
        dq_d = q @ d
        P = P + q - 2.0 * dq_d[:, None] * d                       # read = H m'
        d_dir -= 2.0 * (dq_d[:, None] * m_new + (m_new @ d)[:, None] * q)
        d_cand[:, t] = P * wg[:, t] * (1.0 - c[:, t] ** 2)
        d_write[:, t] = P * c[:, t] * wg[:, t] * (1.0 - wg[:, t])
        mo_d = m_old @ d
        d_decay[:, t] = P * (m_old - 2.0 * mo_d[:, None] * d)
        e = decay * P                                              # dL/dh
        e_d = e @ d
        d_dir -= 2.0 * (e_d[:, None] * m_old + mo_d[:, None] * e)
        P = e - 2.0 * e_d[:, None] * d                             # h = H m
    return tuple(x.astype(np.float32) for x in (d_cand, d_write, d_decay, d_dir, P))
