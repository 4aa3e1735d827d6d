"""Chunked (WY) form of the WKV-7 chunk summary -- TEST INFRASTRUCTURE ONLY.

The WKV-7 recurrence of ``RWKV7TimeMix._torch_recurrence``
(yufmusicgen/model.py:145-165), with S [N, N] (row i = value, column j = key),

    S_t = S_{t-1} G_t + v_t k_t^T,   G_t = diag(w_t) + a_t b_t^T,   y_t = S_t r_t,

is linear in S, so over a chunk of tokens started from S_0

    S_end = S_0 P + U,   y_t = S_0 q_t + yU_t,

with P the chunk's transition, U its end state from a zero start, yU_t the
outputs from a zero start and q_t = P_t r_t.  These four are what the
time-parallel scan's first pass produces and its carry and correction passes
consume.  The scan computes them token by token (7 N^2 FMAs per token); this
module restates them with matrix products over sub-chunks of L tokens, the form
a tensor-core kernel would use.  Inside a sub-chunk, with the cumulative decay
Gamma_t = w_1 ... w_t (elementwise) and the scaled vectors

    a^_t = Gamma_{t-1} a_t,  b^_t = b_t / Gamma_t,  k^_t = k_t / Gamma_t,  r^_t = Gamma_t r_t,

the rows u_t = S_{t-1} a_t satisfy the unit lower-triangular system

    U_rows = A^ S_0^T + tril_strict(A^ B^^T) U_rows + tril_strict(A^ K^^T) V,

so with T = (I - tril_strict(A^ B^^T))^-1, W = T A^ and U0 = T tril_strict(A^ K^^T) V:

    Q_sub  = R^ + tril(R^ B^^T) W                     (rows q_t)
    Y0_sub = tril(R^ B^^T) U0 + tril(R^ K^^T) V       (rows yU_t)
    P_sub  = (I + W^T B^) diag(Gamma_L)
    U_sub  = (U0^T B^ + V^T K^) diag(Gamma_L).

Sub-chunks chain as  q_t = P_cur q_sub,t,  yU_t = U_cur q_sub,t + y0_sub,t,
P_cur <- P_cur P_sub,  U_cur <- U_cur P_sub + U_sub.  The decay is clamped to
w >= exp(-0.6065306597) = 0.545, so 1/Gamma stays below 0.545^-L (2.6e16 for
L = 64), inside the float32 range.

Validated against the reference recurrence in tests/test_wy_form.py; no
product code calls it.
"""

from __future__ import annotations

import numpy as np

from .scans import W_SCALE, _sigmoid


def chunk_summary_wy(r, w_raw, k, v, a, b, sub=16, dtype=np.float64):
    """Chunk summary of one (sequence, head) chunk in the WY form.

    Inputs are [T, N] (T tokens of one head).  Returns
    ``(yU [T, N], Q [T, N], U [N, N], P [N, N])`` with ``y_t = S_0 @ Q[t] +
    yU[t]`` and ``S_end = S_0 @ P + U`` for any start state S_0.
    """
    r, w_raw, k, v, a, b = (np.asarray(x, dtype) for x in (r, w_raw, k, v, a, b))
    T, N = r.shape
    w = np.exp(dtype(W_SCALE) * _sigmoid(w_raw).astype(dtype))
    P_cur = np.eye(N, dtype=dtype)
    U_cur = np.zeros((N, N), dtype)
    yU = np.empty((T, N), dtype)
    Q = np.empty((T, N), dtype)
    for t0 in range(0, T, sub):
        sl = slice(t0, min(t0 + sub, T))
        L = sl.stop - sl.start
        gam = np.cumprod(w[sl], axis=0)                       # Gamma_t, t = 1..L
        gam_prev = np.vstack([np.ones((1, N), dtype), gam[:-1]])
        ah, bh = gam_prev * a[sl], b[sl] / gam
        kh, rh = k[sl] / gam, gam * r[sl]
        strict = np.tril(np.ones((L, L), dtype), -1)
        incl = np.tril(np.ones((L, L), dtype))
        m_ab, m_ak = strict * (ah @ bh.T), strict * (ah @ kh.T)
        m_rb, m_rk = incl * (rh @ bh.T), incl * (rh @ kh.T)
        tinv = np.linalg.solve(np.eye(L, dtype=dtype) - m_ab, np.eye(L, dtype=dtype))
        W = tinv @ ah
        U0 = tinv @ (m_ak @ v[sl])
        q_sub = rh + m_rb @ W
        y0_sub = m_rb @ U0 + m_rk @ v[sl]
        g_end = gam[-1]
        P_sub = (np.eye(N, dtype=dtype) + W.T @ bh) * g_end[None, :]
        U_sub = (U0.T @ bh + v[sl].T @ kh) * g_end[None, :]
        Q[sl] = q_sub @ P_cur.T
        yU[sl] = q_sub @ U_cur.T + y0_sub
        U_cur = U_cur @ P_sub + U_sub
        P_cur = P_cur @ P_sub
    return yU, Q, U_cur, P_cur
