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

Forward only: the training backward of the reference (rwkv7_clampw.cu:83-176)
is not part of this build, so differentiating through ``rwkv7_cuda`` raises.
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


ALGO_AUTO, ALGO_SEQUENTIAL, ALGO_CHUNKED, ALGO_PARALLEL = 0, 1, 2, 3


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


class _RWKV7Function(torch.autograd.Function):
    @staticmethod
    def forward(ctx, r, w, k, v, a, b, state):
        y, s = wkv7_forward(r, w, k, v, a, b, state)
        ctx.mark_non_differentiable(s)
        return y, s

    @staticmethod
    def backward(ctx, grad_y, grad_s):  # pragma: no cover - training is out of scope
        raise NotImplementedError(
            "yufmusicgen_b200 implements the WKV-7 forward only; the training backward "
            "(rwkv7_clampw.cu:83-176) is not part of this build"
        )


def rwkv7_cuda(r, w, k, v, a, b, state=None):
    """Run the fused RWKV-7 recurrence and return output plus final state."""
    if torch.is_grad_enabled() and any(x.requires_grad for x in (r, w, k, v, a, b)):
        return _RWKV7Function.apply(r, w, k, v, a, b, state)
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
