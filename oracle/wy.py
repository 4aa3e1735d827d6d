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


def tf32_round(x):
    """Round float32 values to tf32 (10 explicit mantissa bits, to nearest)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)


def mm_3xtf32(A, B):
    """A @ B as a tensor core computes it with 3xTF32: both operands split into
    a tf32 high part and a tf32-rounded remainder, the products hi.hi + hi.lo +
    lo.hi summed into a float32 accumulator."""
    A = np.asarray(A, np.float32)
    B = np.asarray(B, np.float32)
    ah, bh = tf32_round(A), tf32_round(B)
    al, bl = tf32_round(A - ah), tf32_round(B - bh)
    f = lambda X, Y: X.astype(np.float64) @ Y.astype(np.float64)
    return (f(ah, bh) + f(ah, bl) + f(al, bh)).astype(np.float32)


def unit_lower_inverse_blocked(A, blk, mm):
    """Inverse of a unit lower-triangular A (L x L) with blk x blk diagonal
    blocks inverted by forward substitution and every off-diagonal block formed
    by products:  T_ii = A_ii^-1,  T_ij = -T_ii sum_{k=j..i-1} A_ik T_kj."""
    L = A.shape[0]
    nb = (L + blk - 1) // blk
    T = np.zeros_like(A)
    s = [slice(i * blk, min(L, (i + 1) * blk)) for i in range(nb)]
    for i in range(nb):
        D = A[s[i], s[i]]
        n = D.shape[0]
        Ti = np.zeros_like(D)
        for c in range(n):  # forward substitution on the unit diagonal block
            e = np.zeros(n, A.dtype)
            e[c] = 1
            for r in range(n):
                e[r] -= D[r, :r] @ e[:r] if r > c else 0
            Ti[:, c] = e
        T[s[i], s[i]] = Ti
        for j in range(i):
            acc = sum(mm(A[s[i], s[k]], T[s[k], s[j]]) for k in range(j, i))
            T[s[i], s[j]] = -mm(Ti, acc)
    return T


def chunk_summary_wy_blocked(r, w_raw, k, v, a, b, sub=64, blk=16, mm=mm_3xtf32):
    """The WY chunk summary in the order a tensor-core kernel computes it:
    float32 data, sub-chunks of `sub` tokens, the triangular solve blocked by
    `blk`, and every matrix product done by `mm` (3xTF32 emulation by default).
    Same outputs as chunk_summary_wy."""
    f32 = np.float32
    r, w_raw, k, v, a, b = (np.asarray(x, f32) for x in (r, w_raw, k, v, a, b))
    T, N = r.shape
    w = np.exp(f32(W_SCALE) * _sigmoid(w_raw)).astype(f32)
    P_cur = np.eye(N, dtype=f32)
    U_cur = np.zeros((N, N), f32)
    yU = np.empty((T, N), f32)
    Q = np.empty((T, N), f32)
    for t0 in range(0, T, sub):
        sl = slice(t0, min(t0 + sub, T))
        L = sl.stop - sl.start
        gam = np.cumprod(w[sl], axis=0).astype(f32)
        gam_prev = np.vstack([np.ones((1, N), f32), gam[:-1]])
        ah, bh = gam_prev * a[sl], b[sl] / gam
        kh, rh = k[sl] / gam, gam * r[sl]
        strict = np.tril(np.ones((L, L), f32), -1)
        incl = np.tril(np.ones((L, L), f32))
        m_ab, m_ak = strict * mm(ah, bh.T), strict * mm(ah, kh.T)
        m_rb, m_rk = incl * mm(rh, bh.T), incl * mm(rh, kh.T)
        tinv = unit_lower_inverse_blocked(np.eye(L, dtype=f32) - m_ab, blk, mm)
        W = mm(tinv, ah)
        U0 = mm(tinv, mm(m_ak, v[sl]))
        q_sub = rh + mm(m_rb, W)
        y0_sub = mm(m_rb, U0) + mm(m_rk, v[sl])
        g_end = gam[-1]
        P_sub = (np.eye(N, dtype=f32) + mm(W.T, bh)) * g_end[None, :]
        U_sub = (mm(U0.T, bh) + mm(v[sl].T, kh)) * g_end[None, :]
        Q[sl] = mm(q_sub, P_cur.T)
        yU[sl] = mm(q_sub, U_cur.T) + y0_sub
        U_cur = mm(U_cur, P_sub) + U_sub
        P_cur = mm(P_cur, P_sub)
    return yU, Q, U_cur, P_cur
