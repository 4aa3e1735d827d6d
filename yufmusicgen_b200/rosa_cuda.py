"""Drop-in for ``yufmusicgen/rosa_cuda.py``: the ROSA scan on the B200 kernel.

* ``rosa_householder_scan(cand, write, read_raw, decay, direction, memory)``
  -> ``(read [B,T,R] UNGATED, final_memory [B,R])``, the reference contract
  (rosa_cuda.py:157-180, rosa_householder.cu:89-91): inputs are cast to fp32
  contiguous, ``decay`` is post-sigmoid and ``direction`` a unit vector; the
  caller applies ``sigmoid(read_raw)`` (yufmusicgen/model.py:311).
* ``rosa_cuda_enabled()`` (rosa_cuda.py:69-70).
* Extension: ``rosa_scan(..., gated=True)`` returns the gated read of
  ``ROSAMemory._reference_recurrence`` (yufmusicgen/model.py:260-288) in one
  pass.

Forward only (the reference backward, rosa_householder.cu:103-285, is not
part of this build).
"""

from __future__ import annotations

import os

import torch

from . import _lib


def rosa_cuda_enabled() -> bool:
    return torch.cuda.is_available() and os.environ.get("YUFMUSICGEN_DISABLE_CUDA", "0") != "1"


def rosa_scan(cand, write, read_gate, decay, direction, memory, gated=True, out=None, memory_out=None):
    tensors = (cand, write, read_gate, decay, direction, memory)
    if not all(x.is_cuda for x in tensors):
        raise ValueError("ROSA CUDA inputs must be on CUDA")
    cand, write, read_gate, decay, direction, memory = (x.float().contiguous() for x in tensors)
    if len({tuple(x.shape) for x in (cand, write, read_gate)}) != 1:
        raise ValueError("ROSA CUDA per-step inputs must have identical shapes")
    B, T, R = cand.shape
    if decay.numel() != R or direction.numel() != R or memory.shape != (B, R):
        raise ValueError("ROSA CUDA: decay/direction must be [R] and memory [B, R]")
    read = out if out is not None else torch.empty_like(cand)
    m_out = memory_out if memory_out is not None else torch.empty_like(memory)
    with torch.cuda.device(cand.device):
        stream = torch.cuda.current_stream(cand.device).cuda_stream
        _lib.call("yuf_rosa_forward", _lib.ptr(cand), _lib.ptr(write), _lib.ptr(read_gate),
                  _lib.ptr(decay), _lib.ptr(direction), _lib.ptr(memory), _lib.ptr(read),
                  _lib.ptr(m_out), B, T, R, 1 if gated else 0, stream)
    return read, m_out


def rosa_householder_scan(cand, write, read_raw, decay, direction, memory):
    """Run the fused Householder scan and return ``(read, final_memory)``."""
    if torch.is_grad_enabled() and any(x.requires_grad for x in (cand, write, read_raw, decay, direction, memory)):
        raise NotImplementedError(
            "yufmusicgen_b200 implements the ROSA forward only; the training backward "
            "(rosa_householder.cu:103-285) is not part of this build"
        )
    return rosa_scan(cand, write, read_raw, decay, direction, memory, gated=False)
