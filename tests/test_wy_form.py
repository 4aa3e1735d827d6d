"""The chunked (WY) form of the WKV-7 chunk summary (oracle/wy.py) against the
reference recurrence (oracle/scans.py, pinned to the reference's goldens): the
four outputs the time-parallel scan's passes exchange (zero-start outputs, q
rows, chunk contribution U and transition P) reproduce the token-by-token
scan from any start state, for sub-chunks of 8 to 64 tokens, in float64 and
in float32 (the precision a tensor-core kernel's 3xTF32 products approach).
Tolerance: |got - want| <= 1e-3 + 1e-4 |want|."""

import numpy as np
import pytest

from oracle.scans import wkv7_scan
from oracle.wy import chunk_summary_wy
from yufmusicgen_b200.workloads import wkv_op_inputs

RTOL, ATOL = 1e-4, 1e-3


def _case(T, N, seed):
    ins = wkv_op_inputs(1, T, 1, N, seed=seed, with_state=True)
    x = {k: ins[k][0, :, 0] for k in "rwkvab"}
    s0 = ins["s0"][0, 0]
    y, s = wkv7_scan(*(ins[k] for k in "rwkvab"), ins["s0"])
    return x, s0, y[0, :, 0], s[0, 0]


@pytest.mark.parametrize("sub", [8, 16, 32, 64])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("T,N", [(160, 40), (100, 64), (37, 16)])
def test_wy_chunk_summary_reproduces_the_recurrence(T, N, sub, dtype):
    x, s0, y_ref, s_ref = _case(T, N, seed=T + N + sub)
    yU, Q, U, P = chunk_summary_wy(*(x[k] for k in "rwkvab"), sub=sub, dtype=dtype)
    y = Q @ s0.T.astype(dtype) + yU          # y_t = S_0 q_t + yU_t
    s = s0.astype(dtype) @ P + U             # S_end = S_0 P + U
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(s, s_ref, rtol=RTOL, atol=ATOL)


def test_wy_zero_start_outputs_are_the_scan_from_zero():
    x, _, _, _ = _case(160, 40, seed=7)
    ins = {k: x[k][None, :, None] for k in "rwkvab"}
    y0, s0 = wkv7_scan(*(ins[k] for k in "rwkvab"))
    yU, _, U, _ = chunk_summary_wy(*(x[k] for k in "rwkvab"), sub=16)
    np.testing.assert_allclose(yU, y0[0, :, 0], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(U, s0[0, 0], rtol=RTOL, atol=ATOL)


hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=30, deadline=None, derandomize=True)
@given(T=st.integers(1, 96), N=st.sampled_from([8, 16, 24, 32, 40, 64]),
       sub=st.sampled_from([1, 3, 8, 16, 48]), seed=st.integers(0, 10_000))
def test_wy_form_property_any_shape(T, N, sub, seed):
    """Any chunk length (ragged last sub-chunk included), head size and
    sub-chunk size: the WY summary equals the token-by-token recurrence."""
    x, s0, y_ref, s_ref = _case(T, N, seed)
    yU, Q, U, P = chunk_summary_wy(*(x[k] for k in "rwkvab"), sub=sub)
    np.testing.assert_allclose(Q @ s0.T + yU, y_ref, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(s0 @ P + U, s_ref, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("sub,blk", [(64, 16), (64, 8), (32, 16), (128, 16)])
@pytest.mark.parametrize("T,N", [(160, 40), (128, 64), (70, 16)])
def test_blocked_wy_with_3xtf32_products(T, N, sub, blk):
    """The planned tensor-core schedule: float32 data, 64-token sub-chunks, the
    triangular solve blocked into 16 x 16 diagonal blocks plus products, every
    product a 3xTF32 tensor-core MMA (emulated) -- within the fp32 tolerance."""
    from oracle.wy import chunk_summary_wy_blocked

    x, s0, y_ref, s_ref = _case(T, N, seed=T * 7 + N + sub + blk)
    yU, Q, U, P = chunk_summary_wy_blocked(*(x[k] for k in "rwkvab"), sub=sub, blk=blk)
    np.testing.assert_allclose(Q @ s0.T + yU, y_ref, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(s0 @ P + U, s_ref, rtol=RTOL, atol=ATOL)


def test_blocked_unit_lower_inverse():
    from oracle.wy import mm_3xtf32, unit_lower_inverse_blocked

    rng = np.random.default_rng(3)
    A = np.eye(64, dtype=np.float32) - np.tril(rng.standard_normal((64, 64)).astype(np.float32) * 0.1, -1)
    T = unit_lower_inverse_blocked(A, 16, mm_3xtf32)
    np.testing.assert_allclose(T @ A, np.eye(64), atol=1e-5)
