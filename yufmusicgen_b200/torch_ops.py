"""Register the reference's torch custom ops on the B200 kernels.

After ``import yufmusicgen_b200.torch_ops`` these calls work exactly as the
reference's JIT-built extensions define them:

* ``torch.ops.yufmusicgen_rwkv7.forward(r, w, k, v, a, b, y, state, sa)``
  (rwkv7_clampw.cpp:18-33, 65-68): every output preallocated by the caller and
  filled in place -- ``y [B,T,H,N]``, ``state [B,H,T/16,N,N]`` (the state after
  every 16th token, transposed: ``state[b,h,c,j,i] = S_ij``) and
  ``sa [B,T,H,N]``.  T must be a multiple of 16 (cuda_ops.py pads).
* ``torch.ops.yufmusicgen_rosa.forward(cand, write, read_raw, decay, direction,
  memory, read_out, memory_out, cand_saved, write_saved, read_saved, gate_saved,
  decay_saved, mem_saved)`` (rosa_householder.cpp:24-50, 85-88).

* ``torch.ops.yufmusicgen_rwkv7.backward(r, w, k, v, a, b, dy, state, sa, dr,
  dw, dk, dv, da, db)`` (rwkv7_clampw.cpp:40-63) and
  ``torch.ops.yufmusicgen_rosa.backward(cand_saved, write_saved, read_saved,
  gate_saved, decay_saved, mem_saved, direction, final_memory, d_read, d_cand,
  d_write, d_read_raw, d_decay, d_direction_partial, d_memory_out, workspace)``
  (rosa_householder.cpp:52-83), gradients filled in place.

so ``yufmusicgen/cuda_ops.py`` and ``yufmusicgen/rosa_cuda.py`` run unchanged,
training included, once their ``load(...)`` of the reference extension is
replaced by importing this module.  Do not load the reference extensions in the
same process: the op namespaces would collide.
"""

from __future__ import annotations

import torch

from . import _lib

_RWKV_NS = "yufmusicgen_rwkv7"
_ROSA_NS = "yufmusicgen_rosa"

_libs = []


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _rwkv7_forward(r, w, k, v, a, b, y, state, sa):
    B, T, H, N = r.shape
    with torch.cuda.device(r.device):
        _lib.call("yuf_wkv7_forward_compat", r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(),
                  a.data_ptr(), b.data_ptr(), y.data_ptr(), state.data_ptr(), sa.data_ptr(),
                  B, T, H, N, _stream(r))


def _rosa_forward(cand, write, read_raw, decay, direction, memory, read_out, memory_out,
                  cand_saved, write_saved, read_saved, gate_saved, decay_saved, mem_saved):
    B, T, R = cand.shape
    with torch.cuda.device(cand.device):
        _lib.call("yuf_rosa_forward_compat", *(x.data_ptr() for x in (
            cand, write, read_raw, decay, direction, memory, read_out, memory_out, cand_saved,
            write_saved, read_saved, gate_saved, decay_saved, mem_saved)), B, T, R, _stream(cand))


def _rwkv7_backward(r, w, k, v, a, b, dy, state, sa, dr, dw, dk, dv, da, db):
    B, T, H, N = r.shape
    with torch.cuda.device(r.device):
        _lib.call("yuf_wkv7_backward", *(x.data_ptr() for x in (
            r, w, k, v, a, b, dy, state, sa, dr, dw, dk, dv, da, db)), B, T, H, N, _stream(r))


def _rosa_backward(cand_saved, write_saved, read_saved, gate_saved, decay_saved, mem_saved,
                   direction, final_memory, d_read, d_cand, d_write, d_read_raw, d_decay,
                   d_direction_partial, d_memory_out, workspace):
    B, T, R = cand_saved.shape
    with torch.cuda.device(cand_saved.device):
        _lib.call("yuf_rosa_backward", *(x.data_ptr() for x in (
            cand_saved, write_saved, read_saved, gate_saved, decay_saved, mem_saved, direction,
            final_memory, d_read, d_cand, d_write, d_read_raw, d_decay, d_direction_partial,
            d_memory_out, workspace)), B, T, R, _stream(cand_saved))


def register() -> None:
    """Define and implement both ops (idempotent)."""
    if _libs:
        return
    lib_r = torch.library.Library(_RWKV_NS, "DEF")
    lib_r.define(
        "forward(Tensor r, Tensor w, Tensor k, Tensor v, Tensor a, Tensor b, "
        "Tensor(a!) y, Tensor(b!) state, Tensor(c!) sa) -> ()"
    )
    lib_r.impl("forward", _rwkv7_forward, "CUDA")
    lib_r.define(
        "backward(Tensor r, Tensor w, Tensor k, Tensor v, Tensor a, Tensor b, Tensor dy, "
        "Tensor state, Tensor sa, Tensor(a!) dr, Tensor(b!) dw, Tensor(c!) dk, Tensor(d!) dv, "
        "Tensor(e!) da, Tensor(f!) db) -> ()"
    )
    lib_r.impl("backward", _rwkv7_backward, "CUDA")
    lib_o = torch.library.Library(_ROSA_NS, "DEF")
    lib_o.define(
        "forward(Tensor cand, Tensor write, Tensor read_raw, Tensor decay, Tensor direction, "
        "Tensor memory, Tensor(a!) read_out, Tensor(b!) memory_out, Tensor(c!) cand_saved, "
        "Tensor(d!) write_saved, Tensor(e!) read_saved, Tensor(f!) gate_saved, "
        "Tensor(g!) decay_saved, Tensor(h!) mem_saved) -> ()"
    )
    lib_o.impl("forward", _rosa_forward, "CUDA")
    lib_o.define(
        "backward(Tensor cand_saved, Tensor write_saved, Tensor read_saved, Tensor gate_saved, "
        "Tensor decay_saved, Tensor mem_saved, Tensor direction, Tensor final_memory, "
        "Tensor d_read, Tensor(a!) d_cand, Tensor(b!) d_write, Tensor(c!) d_read_raw, "
        "Tensor(d!) d_decay, Tensor(e!) d_direction_partial, Tensor(f!) d_memory_out, "
        "Tensor(g!) workspace) -> ()"
    )
    lib_o.impl("backward", _rosa_backward, "CUDA")
    _libs.extend([lib_r, lib_o])


register()
