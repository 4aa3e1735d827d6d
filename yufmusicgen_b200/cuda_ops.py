"""Drop-in for ``yufmusicgen/cuda_ops.py``: the WKV-7 op on the B200 kernels.

Same public names and behaviour as the reference module:

* ``rwkv7_cuda(r, w, k, v, a, b)`` -> ``(y [B,T,H,N], final_state [B,H,N,N])``
  with the reference's validation errors (cuda_ops.py:200-209) and its final
  state layout: canonical ``S[b,h,i,j]`` (row i = value, col j = key), i.e.
  what ``states[:, :, -1].transpose(-1, -2)`` gives in cuda_ops.py:231.
  Extension: an optional ``state`` (initial state), which the reference op
  cannot take (rwkv7_clampw.cu:25-29), and any T (no padding to 16).
* ``cuda_kernel_enabled()`` / ``report_cuda_fallback(exc)`` (cuda_ops.py:269-283).
* ``CHUNK_LENGTH = 16``.

Training: with inputs that require grad, ``rwkv7_cuda`` runs the reference's
op contract (T padded to 16, checkpoints and sa saved) and its backward runs
``yuf_wkv7_backward`` (the reference's rwkv7_clampw.cu:83-176 contract).
"""

from __future__ import annotations

import os
import warnings

import torch

from . import _lib

CHUNK_LENGTH = 16
_WARNED = False


def _validate(tensors, names=("r", "w", "k", "v", "a", "b")):
    r = tensors[0]
    if r.ndim != 4:
        raise ValueError("RWKV-7 CUDA inputs must have shape [B, T, H, N]")
    if not all(x.is_cuda for x in tensors):
        raise ValueError("RWKV-7 CUDA inputs must be on CUDA")
    if not all(x.dtype == torch.float32 for x in tensors):
        raise TypeError("the bundled default kernel is compiled for float32")
    if not all(x.is_contiguous() for x in tensors):
        raise ValueError("RWKV-7 CUDA inputs must be contiguous")
    if len({tuple(x.shape) for x in tensors}) != 1:
        raise ValueError("RWKV-7 CUDA inputs must have identical shapes")
    if len({x.device for x in tensors}) != 1:
        raise ValueError("RWKV-7 CUDA inputs must be on one device")


ALGO_AUTO, ALGO_SEQUENTIAL, ALGO_CHUNKED, ALGO_PARALLEL, ALGO_PARALLEL_TC, ALGO_ROWS, ALGO_CHUNKED_TC = range(7)


def wkv7_forward(r, w, k, v, a, b, state=None, out=None, state_out=None, algo=ALGO_AUTO):
    """Raw WKV-7 forward through ``yuf_wkv7_forward_ex``; returns (y, final_state).

    ``state`` is the [B,H,N,N] initial state or None (zeros).  ``state_out``
    may be ``state`` itself (updated in place).  ``algo`` picks the sequential
    (token by token) or chunked kernel; AUTO uses the single-token decode
    kernel for T == 1 and the sequential kernel otherwise."""
    _validate((r, w, k, v, a, b))
    B, T, H, N = r.shape
    if state is not None:
        if state.shape != (B, H, N, N) or state.dtype != torch.float32 or not state.is_contiguous():
            raise ValueError("state must be a contiguous float32 [B, H, N, N] tensor")
        if state.device != r.device:
            raise ValueError("state must be on the inputs' device")
    y = out if out is not None else torch.empty_like(r)
    s_out = state_out if state_out is not None else torch.empty((B, H, N, N), device=r.device, dtype=torch.float32)
    with torch.cuda.device(r.device):
        stream = torch.cuda.current_stream(r.device).cuda_stream
        _lib.call("yuf_wkv7_forward_ex", _lib.ptr(r), _lib.ptr(w), _lib.ptr(k), _lib.ptr(v),
                  _lib.ptr(a), _lib.ptr(b), _lib.ptr(state), _lib.ptr(y), _lib.ptr(s_out),
                  B, T, H, N, algo, stream)
    return y, s_out


def wkv7_forward_compat(r, w, k, v, a, b, y=None, states=None, sa=None):
    """The reference op's forward contract (``yuf_wkv7_forward_compat``): zero
    initial state, T % 16 == 0; returns ``(y, states [B,H,T/16,N,N] transposed
    checkpoints, sa [B,T,H,N])``."""
    _validate((r, w, k, v, a, b))
    B, T, H, N = r.shape
    y = torch.empty_like(r) if y is None else y
    states = torch.empty(B, H, T // CHUNK_LENGTH, N, N, device=r.device) if states is None else states
    sa = torch.empty_like(r) if sa is None else sa
    with torch.cuda.device(r.device):
        _lib.call("yuf_wkv7_forward_compat", *(_lib.ptr(x) for x in (r, w, k, v, a, b, y, states, sa)),
                  B, T, H, N, torch.cuda.current_stream(r.device).cuda_stream)
    return y, states, sa


def wkv7_backward(r, w, k, v, a, b, dy, states, sa, grads=None):
    """Gradients ``(dr, dw, dk, dv, da, db)`` of the compat forward
    (``yuf_wkv7_backward``; rwkv7_clampw.cpp:40-63)."""
    _validate((r, w, k, v, a, b, dy, sa))
    B, T, H, N = r.shape
    grads = [torch.empty_like(r) for _ in range(6)] if grads is None else grads
    with torch.cuda.device(r.device):
        _lib.call("yuf_wkv7_backward", *(_lib.ptr(x) for x in (r, w, k, v, a, b, dy, states, sa)),
                  *(_lib.ptr(g) for g in grads), B, T, H, N,
                  torch.cuda.current_stream(r.device).cuda_stream)
    return tuple(grads)


def _pad16(r, w, k, v, a, b):
    """Pad T to a multiple of 16 as cuda_ops.py:159-186 does: zero r/k/v/a/b and
    w_raw = -80 (retention 1), so the padded steps leave the state unchanged."""
    T = r.shape[1]
    extra = (-T) % CHUNK_LENGTH
    if extra == 0:
        return (r, w, k, v, a, b), T
    def pad(x, value):
        tail = torch.full((x.shape[0], extra, *x.shape[2:]), value, device=x.device, dtype=x.dtype)
        return torch.cat((x, tail), dim=1).contiguous()
    return (pad(r, 0.0), pad(w, -80.0), pad(k, 0.0), pad(v, 0.0), pad(a, 0.0), pad(b, 0.0)), T


class _RWKV7Function(torch.autograd.Function):
    """Differentiable op: the compat forward saves the 16-token checkpoints and
    sa, the backward kernel consumes them (the reference's _RWKV7CUDAFunction,
    cuda_ops.py:189-253).  Zero initial state only, as in the reference."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b):
        (rp, wp, kp, vp, ap, bp), T = _pad16(r, w, k, v, a, b)
        y, states, sa = wkv7_forward_compat(rp, wp, kp, vp, ap, bp)
        ctx.save_for_backward(rp, wp, kp, vp, ap, bp, states, sa)
        ctx.T = T
        final_state = states[:, :, -1].transpose(-1, -2).contiguous()
        ctx.mark_non_differentiable(final_state)
        return y[:, :T].contiguous(), final_state

    @staticmethod
    def backward(ctx, grad_y, grad_s):
        rp, wp, kp, vp, ap, bp, states, sa = ctx.saved_tensors
        dy = torch.zeros_like(rp)
        dy[:, :ctx.T] = grad_y
        grads = wkv7_backward(rp, wp, kp, vp, ap, bp, dy, states, sa)
        return tuple(g[:, :ctx.T].contiguous() for g in grads)


def rwkv7_cuda(r, w, k, v, a, b, state=None):
    """Run the fused RWKV-7 recurrence and return output plus final state.
    Differentiable (zero initial state) when an input requires grad."""
    if torch.is_grad_enabled() and any(x.requires_grad for x in (r, w, k, v, a, b)):
        if state is not None:
            raise NotImplementedError(
                "rwkv7_cuda: gradients need a zero initial state (the reference op has no state input)")
        _validate((r, w, k, v, a, b))
        return _RWKV7Function.apply(r, w, k, v, a, b)
    return wkv7_forward(r, w, k, v, a, b, state)


def cuda_kernel_enabled() -> bool:
    return torch.cuda.is_available() and os.environ.get("YUFMUSICGEN_DISABLE_CUDA", "0") != "1"


def report_cuda_fallback(exc: Exception) -> None:
    global _WARNED
    if _WARNED or os.environ.get("YUFMUSICGEN_SILENCE_CUDA_WARNING", "0") == "1":
        return
    _WARNED = True
    warnings.warn(
        "YufMusicGen RWKV-7 CUDA kernel unavailable; using the PyTorch recurrence. "
        f"Reason: {exc}",
        RuntimeWarning,
        stacklevel=3,
    )
