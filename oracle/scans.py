"""numpy restatement of the two recurrences on the hot path (test oracle).

Both functions follow the reference's PyTorch loops step by step, with the
same operation order, in float32.
"""

from __future__ import annotations

import numpy as np

W_SCALE = np.float32(-0.6065306597)  # yufmusicgen/model.py:156


def _sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def wkv7_scan(r, w_raw, k, v, a, b, s0=None):
    """``RWKV7TimeMix._torch_recurrence`` (yufmusicgen/model.py:145-165).

    Inputs are [B, T, H, N] float32; ``s0`` is [B, H, N, N] (row i = value
    dim, column j = key dim) or None for a zero state.  Returns
    ``(y [B, T, H, N], s_T [B, H, N, N])``.
    """
    r, w_raw, k, v, a, b = (np.asarray(x, np.float32) for x in (r, w_raw, k, v, a, b))
    B, T, H, N = r.shape
    S = np.zeros((B, H, N, N), np.float32) if s0 is None else np.array(s0, np.float32, copy=True)
    retention = np.exp(W_SCALE * _sigmoid(w_raw)).astype(np.float32)
    y = np.empty((B, T, H, N), np.float32)
    for t in range(T):
        sa = np.einsum("bhj,bhij->bhi", a[:, t], S)
        S = (
            S * retention[:, t][:, :, None, :]
            + sa[..., None] * b[:, t][:, :, None, :]
            + v[:, t][..., None] * k[:, t][:, :, None, :]
        ).astype(np.float32)
        y[:, t] = np.einsum("bhij,bhj->bhi", S, r[:, t])
    return y, S


def rosa_scan(cand, write, read_gate, decay, direction, m0):
    """``ROSAMemory._reference_recurrence`` (yufmusicgen/model.py:260-288).

    ``decay`` is post-sigmoid [R]; ``direction`` is unit [R]; ``m0`` [B, R].
    Returns ``(read [B, T, R] -- gated by sigmoid(read_gate), m_T [B, R])``.
    """
    cand, write, read_gate = (np.asarray(x, np.float32) for x in (cand, write, read_gate))
    decay = np.asarray(decay, np.float32).reshape(-1)
    d = np.asarray(direction, np.float32).reshape(-1)
    m = np.array(m0, np.float32, copy=True)
    B, T, R = cand.shape
    out = np.empty((B, T, R), np.float32)
    for t in range(T):
        rotated = m - 2.0 * np.sum(m * d, axis=-1, keepdims=True) * d
        m = (decay * rotated + _sigmoid(write[:, t]) * np.tanh(cand[:, t])).astype(np.float32)
        read = m - 2.0 * np.sum(m * d, axis=-1, keepdims=True) * d
        out[:, t] = read * _sigmoid(read_gate[:, t])
    return out, m


def rosa_scan_ungated(cand, write, read_gate, decay, direction, m0):
    """The reference CUDA op's contract (yufmusicgen/cuda/rosa_householder.cu:30-101):
    the same recurrence, returning the UNGATED read; the caller applies
    ``sigmoid(read_gate)`` (yufmusicgen/model.py:311)."""
    cand, write = (np.asarray(x, np.float32) for x in (cand, write))
    decay = np.asarray(decay, np.float32).reshape(-1)
    d = np.asarray(direction, np.float32).reshape(-1)
    m = np.array(m0, np.float32, copy=True)
    B, T, R = cand.shape
    out = np.empty((B, T, R), np.float32)
    for t in range(T):
        rotated = m - 2.0 * np.sum(m * d, axis=-1, keepdims=True) * d
        m = (decay * rotated + _sigmoid(write[:, t]) * np.tanh(cand[:, t])).astype(np.float32)
        out[:, t] = m - 2.0 * np.sum(m * d, axis=-1, keepdims=True) * d
    return out, m
