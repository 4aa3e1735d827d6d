"""On-device sampling (C ABI ``yuf_sample``), the GPU counterpart of the
reference's host-side ``sample_token`` and masking (yufmusicgen/cli/generate.py:45-56,
142-149).  The random stream is Philox4x32-10 keyed by ``seed`` with counter
(step, sequence), so draws are reproducible and independent of batching.
"""

from __future__ import annotations

import torch

from . import _lib
from .config import EOS, MIDI_OFFSET


def sample(logits, seed: int, step: int, temperature: float = 1.0, top_k: int = 32,
           top_p: float = 1.0, seq0: int = 0, mask_below: int = 0, eos_id: int = EOS,
           allow_eos: bool = True, out=None, return_uniform: bool = False):
    """Sample one id per row of ``logits`` [B, V] (CUDA fp32)."""
    if logits.dtype != torch.float32 or not logits.is_cuda or logits.ndim != 2:
        raise ValueError("logits must be a CUDA float32 [B, V] tensor")
    logits = logits.contiguous()
    B, V = logits.shape
    ids = out if out is not None else torch.empty(B, dtype=torch.int32, device=logits.device)
    u = torch.empty(B, device=logits.device) if return_uniform else None
    with torch.cuda.device(logits.device):
        _lib.call("yuf_sample", logits.data_ptr(), B, V, float(temperature), int(top_k), float(top_p),
                  int(seed) & (2**64 - 1), int(step) & (2**64 - 1), int(seq0), int(mask_below),
                  int(eos_id), 1 if allow_eos else 0, ids.data_ptr(),
                  u.data_ptr() if u is not None else None,
                  torch.cuda.current_stream(logits.device).cuda_stream)
    return (ids, u) if return_uniform else ids


def sample_music(logits, seed: int, step: int, generated: int, temperature: float = 1.0,
                 top_k: int = 32, top_p: float = 1.0, seq0: int = 0, out=None):
    """The reference generation loop's rule: only MIDI ids, and EOS once at least
    16 tokens were generated (generate.py:142-147)."""
    return sample(logits, seed, step, temperature, top_k, top_p, seq0, mask_below=MIDI_OFFSET,
                  eos_id=EOS, allow_eos=generated >= 16, out=out)


def philox_uniform(seed: int, step: int, seq0: int, n: int, device="cuda"):
    out = torch.empty(n, device=device)
    _lib.call("yuf_philox_uniform", int(seed) & (2**64 - 1), int(step) & (2**64 - 1), int(seq0), n,
              out.data_ptr(), torch.cuda.current_stream(out.device).cuda_stream)
    return out


class TorchCpuGenerator:
    """Host generator with the reference's random stream (C ABI ``yuf_mt19937_*``):
    the state of torch's CPU generator after ``torch.manual_seed(seed)``, which
    the reference's generation loop samples from (yufmusicgen/training.py:23-28,
    cli/generate.py:45-56)."""

    def __init__(self, seed: int):
        import ctypes

        self._h = ctypes.c_void_p()
        _lib.call("yuf_mt19937_create", int(seed) & (2**64 - 1), ctypes.byref(self._h))

    def close(self):
        if self._h:
            _lib.call("yuf_mt19937_destroy", self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def next_u32(self, n: int):
        import numpy as np

        out = np.empty(n, np.uint32)
        _lib.call("yuf_mt19937_next", self._h, out.ctypes.data, n)
        return out

    def exponential(self, n: int):
        import numpy as np

        out = np.empty(n, np.float32)
        _lib.call("yuf_mt19937_exponential", self._h, out.ctypes.data, n)
        return out

    def sample(self, logits, temperature: float = 1.0, top_p: float = 0.95):
        """The reference's ``sample_token`` on host logits [B, V] (or [V]); rows
        draw one after another."""
        import numpy as np

        x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        one = x.ndim == 1
        x = x.reshape(1, -1) if one else x
        out = np.empty(x.shape[0], np.int32)
        _lib.call("yuf_sample_host", x.ctypes.data, x.shape[0], x.shape[1], float(temperature),
                  float(top_p), self._h, out.ctypes.data)
        return int(out[0]) if one else out


def mask_like_reference(logits, step: int, mask_below: int = MIDI_OFFSET, eos_id: int = EOS,
                        min_before_eos: int = 16):
    """The reference loop's masking (generate.py:142-147) on host logits [B, V]:
    ids below MIDI_OFFSET become -inf, EOS stays selectable from step 16 on."""
    import numpy as np

    x = np.array(logits, dtype=np.float32, copy=True)
    keep_eos = x[..., eos_id].copy()
    x[..., :mask_below] = -np.inf
    if step >= min_before_eos:
        x[..., eos_id] = keep_eos
    return x
