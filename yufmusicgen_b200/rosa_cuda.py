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

Training: with inputs that require grad, ``rosa_householder_scan`` saves the
reference op's tensors and its backward runs ``yuf_rosa_backward`` (the
contract of rosa_householder.cu:103-285, with the exact gradient).
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


def rosa_forward_compat(cand, write, read_raw, decay, direction, memory):
    """``yuf_rosa_forward_compat``: ungated read, final memory and the saved
    tensors of the reference op (rosa_cuda.py:73-114)."""
    B, T, R = cand.shape
    read_out = torch.empty_like(cand)
    memory_out = torch.empty_like(memory)
    saved = [torch.empty_like(cand) for _ in range(5)]  # cand, write, read, gate, decay
    mem_saved = torch.empty(B, T + 1, R, device=cand.device)
    with torch.cuda.device(cand.device):
        _lib.call("yuf_rosa_forward_compat", *(_lib.ptr(x) for x in (
            cand, write, read_raw, decay, direction, memory, read_out, memory_out, *saved, mem_saved)),
            B, T, R, torch.cuda.current_stream(cand.device).cuda_stream)
    return read_out, memory_out, saved, mem_saved


def rosa_backward(cand_saved, write_saved, read_saved, gate_saved, decay_saved, mem_saved, direction,
                  memory_out, d_read):
    """``yuf_rosa_backward`` (rosa_householder.cpp:52-83): returns d_cand, d_write,
    d_read_raw (zero), d_decay [B,T,R], d_direction_partial [B,R], d_memory [B,R]."""
    B, T, R = cand_saved.shape
    d_read = d_read.float().contiguous()
    outs = [torch.empty_like(cand_saved) for _ in range(4)]
    d_dir = torch.empty(B, R, device=cand_saved.device)
    d_mem = torch.empty(B, R, device=cand_saved.device)
    with torch.cuda.device(cand_saved.device):
        _lib.call("yuf_rosa_backward", *(_lib.ptr(x) for x in (
            cand_saved, write_saved, read_saved, gate_saved, decay_saved, mem_saved, direction,
            memory_out, d_read, *outs, d_dir, d_mem)), None, B, T, R,
            torch.cuda.current_stream(cand_saved.device).cuda_stream)
    return (*outs, d_dir, d_mem)


class _ROSAFunction(torch.autograd.Function):
    """The reference's _ROSAHouseholderFunction (rosa_cuda.py:73-154) on this
    build's kernels; the final memory is non-differentiable, as there."""

    @staticmethod
    def forward(ctx, cand, write, read_raw, decay, direction, memory):
        read_out, memory_out, saved, mem_saved = rosa_forward_compat(
            cand, write, read_raw, decay, direction, memory)
        ctx.save_for_backward(*saved, mem_saved, direction, memory_out)
        ctx.mark_non_differentiable(memory_out)
        return read_out, memory_out

    @staticmethod
    def backward(ctx, d_read, _d_memory_out):
        cs, ws, rs, gs, ds, ms, direction, memory_out = ctx.saved_tensors
        d_cand, d_write, d_read_raw, d_decay, d_dir, d_mem = rosa_backward(
            cs, ws, rs, gs, ds, ms, direction, memory_out, d_read)
        return d_cand, d_write, d_read_raw, d_decay.sum(dim=(0, 1)), d_dir.sum(dim=0), d_mem


def rosa_householder_scan(cand, write, read_raw, decay, direction, memory):
    """Run the fused Householder scan and return ``(read, final_memory)``.
    Differentiable when an input requires grad (R in the reference's
    {16, 32, 64, 128, 256})."""
    if torch.is_grad_enabled() and any(x.requires_grad for x in (cand, write, read_raw, decay, direction, memory)):
        tensors = (cand, write, read_raw, decay, direction, memory)
        if not all(x.is_cuda for x in tensors):
            raise ValueError("ROSA CUDA inputs must be on CUDA")
        cand, write, read_raw, decay, direction, memory = (x.float().contiguous() for x in tensors)
        if len({tuple(x.shape) for x in (cand, write, read_raw)}) != 1:
            raise ValueError("ROSA CUDA per-step inputs must have identical shapes")
        return _ROSAFunction.apply(cand, write, read_raw, decay, direction, memory)
    return rosa_scan(cand, write, read_raw, decay, direction, memory, gated=False)
