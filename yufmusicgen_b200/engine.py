"""Python host API of the model engine (C ABI ``yuf_model_*`` / ``yuf_prefill`` /
``yuf_step`` in include/yufb200.h).

* :class:`Engine` -- batched prefill and decode over device-resident state
  slots; the GPU counterpart of ``YufMusicGen.forward`` / ``.step``
  (yufmusicgen/model.py:406-431) with the state kept on the device.
* :class:`Model` -- single-sequence facade with the Vulkan engine's API
  (``Model::new`` / ``step(token) -> logits`` / ``reset_state``,
  vulkan/src/compute/model.rs:24-65).

All compute runs in ``libyufb200.so``; a missing library or a failing call
raises.  Tensors passed in are torch CUDA tensors (torch is only used here for
device memory and streams).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .config import ModelConfig

PRECISIONS = {"fp32": 0, "bf16": 1}


def _cfg_struct(cfg: ModelConfig) -> _lib.ModelConfigC:
    return _lib.ModelConfigC(cfg.vocab_size, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.head_size,
                             cfg.rosa_size, cfg.low_rank)


class Engine:
    def __init__(self, cfg: ModelConfig | None = None, weights: dict | None = None,
                 precision: str = "fp32", device: int = 0, n_slots: int = 1,
                 yuf_path: str | None = None):
        self._lib = _lib.load()
        self.device = torch.device("cuda", device)
        self.precision = precision
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            if yuf_path is not None:
                _lib.call("yuf_model_create_from_yuf", str(yuf_path).encode(), PRECISIONS[precision],
                          device, ctypes.byref(handle))
                c = _lib.ModelConfigC()
                _lib.call("yuf_model_get_config", handle, ctypes.byref(c))
                cfg = ModelConfig(vocab_size=c.vocab_size, d_model=c.d_model, n_layers=c.n_layers,
                                  n_heads=c.n_heads, head_size=c.head_size, rosa_size=c.rosa_size)
                self.low_rank = c.low_rank
            else:
                if cfg is None or weights is None:
                    raise ValueError("Engine needs (cfg, weights) or yuf_path")
                arrs = {k: np.ascontiguousarray(np.asarray(v, dtype=np.float32)) for k, v in weights.items()}
                names = list(arrs)
                c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
                c_data = (ctypes.c_void_p * len(names))(*[arrs[n].ctypes.data for n in names])
                c_num = (ctypes.c_int64 * len(names))(*[arrs[n].size for n in names])
                cs = _cfg_struct(cfg)
                _lib.call("yuf_model_create", ctypes.byref(cs), PRECISIONS[precision], device, len(names),
                          c_names, c_data, c_num, ctypes.byref(handle))
                self.low_rank = cfg.low_rank
        self.cfg = cfg
        self._h = handle
        self.n_slots = 0
        self.alloc_state(n_slots)

    # -- lifecycle -------------------------------------------------------
    def close(self):
        if self._h:
            _lib.call("yuf_model_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    # -- state -----------------------------------------------------------
    def alloc_state(self, n_slots: int):
        with torch.cuda.device(self.device):
            _lib.call("yuf_state_alloc", self._h, n_slots)
        self.n_slots = n_slots

    def reset_state(self, slot0: int = 0, n: int | None = None):
        n = self.n_slots - slot0 if n is None else n
        with torch.cuda.device(self.device):
            _lib.call("yuf_state_reset", self._h, slot0, n, self._stream())

    def export_state(self, layer: int, slot0: int, n: int):
        c = self.cfg
        prev = torch.empty(n, c.d_model, device=self.device)
        S = torch.empty(n, c.n_heads, c.head_size, c.head_size, device=self.device)
        m = torch.empty(n, c.rosa_size, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("yuf_state_export", self._h, layer, slot0, n, prev.data_ptr(), S.data_ptr(),
                      m.data_ptr(), self._stream())
        return {"prev": prev, "S": S, "m": m}

    def import_state(self, layer: int, slot0: int, prev, S, m):
        n = prev.shape[0]
        with torch.cuda.device(self.device):
            _lib.call("yuf_state_import", self._h, layer, slot0, n, prev.contiguous().data_ptr(),
                      S.contiguous().data_ptr(), m.contiguous().data_ptr(), self._stream())

    # -- compute ---------------------------------------------------------
    def _ids(self, ids):
        t = ids if isinstance(ids, torch.Tensor) else torch.as_tensor(np.asarray(ids))
        return t.to(self.device, dtype=torch.int32).contiguous()

    def prefill(self, ids, slot0: int = 0, all_logits: bool = False, out_last=None, out_all=None):
        """Run ids [B,T] from the state in slots [slot0, slot0+B); returns
        logits of the last token [B,V] (and all logits [B,T,V] if asked)."""
        ids = self._ids(ids)
        B, T = ids.shape
        V = self.cfg.vocab_size
        last = out_last if out_last is not None else torch.empty(B, V, device=self.device)
        allv = None
        if all_logits:
            allv = out_all if out_all is not None else torch.empty(B, T, V, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("yuf_prefill", self._h, ids.data_ptr(), B, T, slot0, last.data_ptr(),
                      allv.data_ptr() if allv is not None else None, self._stream())
        return (last, allv) if all_logits else last

    def step(self, ids, slot0: int = 0, out=None):
        """One decode step: ids [B] -> logits [B,V] for slots [slot0, slot0+B)."""
        ids = self._ids(ids).reshape(-1)
        B = ids.shape[0]
        logits = out if out is not None else torch.empty(B, self.cfg.vocab_size, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("yuf_step", self._h, ids.data_ptr(), B, slot0, logits.data_ptr(), self._stream())
        return logits

    def generate(self, prompt_ids, n_steps: int, temperature: float = 1.0, top_k: int = 32,
                 top_p: float = 1.0, seed: int = 0, seq0: int = 0, mask_below: int = 0,
                 eos_id: int = -1, min_tokens_before_eos: int = 16, slot0: int = 0,
                 reset: bool = True, out_tokens=None, out_lengths=None):
        """Generate ``n_steps`` tokens per sequence on the device (C ABI
        ``yuf_generate``): the batched decode loop of the reference's
        ``run_generation`` (yufmusicgen/cli/generate.py:130-154).

        ``prompt_ids`` [B, T] is prefilled into slots [slot0, slot0 + B), zeroed
        first when ``reset`` (a fresh sequence, as the reference starts from no
        state).  Returns (tokens [B, n_steps], lengths [B]) as device int32
        tensors: a sequence ends at its first ``eos_id`` (not emitted; later
        entries are ``eos_id``), ``lengths`` counts the tokens before it.  The
        reference's own rule is ``mask_below=MIDI_OFFSET, eos_id=EOS,
        min_tokens_before_eos=16`` (generate.py:142-147)."""
        ids = self._ids(prompt_ids)
        B, T = ids.shape
        toks = out_tokens if out_tokens is not None else torch.empty(B, n_steps, dtype=torch.int32,
                                                                     device=self.device)
        lens = out_lengths if out_lengths is not None else torch.empty(B, dtype=torch.int32,
                                                                       device=self.device)
        p = _lib.GenerateParamsC(float(temperature), int(top_k), float(top_p),
                                 int(seed) & (2**64 - 1), int(seq0), int(mask_below), int(eos_id),
                                 int(min_tokens_before_eos))
        if reset:
            self.reset_state(slot0, B)
        with torch.cuda.device(self.device):
            _lib.call("yuf_generate", self._h, ids.data_ptr(), B, T, slot0, int(n_steps),
                      ctypes.byref(p), toks.data_ptr(), lens.data_ptr(), self._stream())
        return toks, lens

    def generate_reference_stream(self, prompt_ids, n_steps: int, temperature: float = 1.0,
                                  top_p: float = 0.95, seed: int = 1337, mask_below: int = 260,
                                  eos_id: int = 2, min_tokens_before_eos: int = 16, slot0: int = 0):
        """The reference's sampled decode with the reference's random stream:
        the loop of run_generation (yufmusicgen/cli/generate.py:130-154) --
        mask to MIDI ids (and EOS from step ``min_tokens_before_eos`` on),
        ``sample_token``'s temperature / top-p rule, ``torch.multinomial`` on the
        CPU generator after ``torch.manual_seed(seed)`` (host MT19937,
        ``yuf_sample_host``), stop at EOS -- so a fixed seed yields the tokens
        the reference's CPU loop draws.  Each step copies the logits to the host
        (the reference synchronises per token too).  One sequence per call, as
        the reference generates; returns the generated ids (EOS not included)."""
        import numpy as np

        from .sampler import TorchCpuGenerator, mask_like_reference

        ids = self._ids(prompt_ids)
        if ids.shape[0] != 1:
            raise ValueError("the reference's loop generates one sequence at a time")
        gen = TorchCpuGenerator(seed)
        self.reset_state(slot0, 1)
        logits = self.prefill(ids, slot0=slot0)
        out = []
        tok = torch.empty(1, dtype=torch.int32, device=self.device)
        try:
            for step in range(n_steps):
                row = mask_like_reference(logits.cpu().numpy(), step, mask_below, eos_id,
                                          min_tokens_before_eos)
                t = int(gen.sample(row, temperature, top_p)[0])
                if t == eos_id:
                    break
                out.append(t)
                tok.fill_(t)
                logits = self.step(tok, slot0=slot0)
        finally:
            gen.close()
        return np.asarray(out, np.int64)

    def set_decode_graphs(self, enabled: bool = True):
        """Replay decode steps as CUDA graphs (needs a non-default stream)."""
        _lib.call("yuf_model_set_decode_graphs", self._h, 1 if enabled else 0)

    def sync_check(self):
        with torch.cuda.device(self.device):
            _lib.call("yuf_model_sync_check", self._h, self._stream())

    # -- parity dumps ----------------------------------------------------
    def set_debug(self, enabled: bool = True, regions=None, layers=None):
        """Keep per-layer parity dumps of every call (all regions and layers, or
        only the named ``regions`` of the given ``layers``)."""
        names = ",".join(regions).encode() if regions else None
        lay = list(layers) if layers else []
        arr = (ctypes.c_int * max(1, len(lay)))(*lay)
        _lib.call("yuf_model_set_debug_filter", self._h, names, arr if lay else None, len(lay))
        _lib.call("yuf_model_set_debug", self._h, 1 if enabled else 0)

    def debug_dump(self, region: str, layer: int = -1) -> np.ndarray:
        n = ctypes.c_size_t()
        _lib.call("yuf_debug_dump", self._h, region.encode(), layer, None, 0, ctypes.byref(n))
        out = np.empty(n.value, np.float32)
        _lib.call("yuf_debug_dump", self._h, region.encode(), layer, out.ctypes.data, out.size,
                  ctypes.byref(n))
        return out


class Model:
    """Single-sequence API of the Vulkan engine (vulkan/src/compute/model.rs:24-65)."""

    def __init__(self, cfg=None, weights=None, precision="fp32", device=0, yuf_path=None):
        self.engine = Engine(cfg, weights, precision, device, n_slots=1, yuf_path=yuf_path)
        self.config = self.engine.cfg

    @classmethod
    def from_yuf(cls, path, precision="fp32", device=0):
        return cls(yuf_path=path, precision=precision, device=device)

    def step(self, token: int) -> list[float]:
        """Run one token; return the vocab-sized logits (Model::step)."""
        logits = self.engine.step(torch.tensor([token], dtype=torch.int32))
        return logits[0].tolist()

    def reset_state(self) -> None:
        """Zero the recurrent state (Model::reset_state)."""
        self.engine.reset_state(0, 1)
