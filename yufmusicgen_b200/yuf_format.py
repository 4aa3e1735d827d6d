"""The ``.yuf`` checkpoint container (writer and reader).

Layout, as ``vulkan/scripts/export_checkpoint.py:47-146`` writes it and
``vulkan/src/checkpoint.rs:90-149`` reads it::

    b"YUFM" | version u32 LE (1) | header_len u64 LE | JSON header | f32 LE data

The JSON header holds ``model_config``, ``tensors`` (``name``, ``shape``,
``offset`` in floats into the data, ``count``) and ``lm_head_alias``; a tied
``lm_head.weight`` is dropped.  Tensor order: embedding, then blocks by layer,
then the final norm (the exporter's ``sort_key``).  ``midi`` / ``source`` are
carried through when given.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

MAGIC = b"YUFM"
VERSION = 1


def _order(name: str):
    if name == "token_embedding.weight":
        return (0, 0)
    if name == "final_norm.weight":
        return (2, 0)
    if name == "final_norm.bias":
        return (2, 1)
    parts = name.split(".")
    return (1, int(parts[1]) if parts[0] == "blocks" else -1)


def write_yuf(path, cfg, weights: dict, midi: dict | None = None, source: dict | None = None) -> None:
    state = dict(weights)
    alias = None
    if getattr(cfg, "tie_embeddings", True) and "lm_head.weight" in state:
        alias = "token_embedding.weight"
        state.pop("lm_head.weight")
    names = sorted(state, key=_order)  # stable: keeps insertion order within a layer
    tensors, chunks, off = [], [], 0
    for n in names:
        a = np.ascontiguousarray(np.asarray(state[n], dtype=np.float32))
        tensors.append({"name": n, "shape": list(a.shape), "offset": off, "count": int(a.size)})
        chunks.append(a.reshape(-1).astype("<f4").tobytes())
        off += a.size
    header = {
        "format": "yufmusicgen-checkpoint",
        "version": VERSION,
        "model_config": {
            "vocab_size": cfg.vocab_size, "d_model": cfg.d_model, "n_layers": cfg.n_layers,
            "n_heads": cfg.n_heads, "head_size": cfg.head_size, "rosa_size": cfg.rosa_size,
            "dropout": getattr(cfg, "dropout", 0.0), "tie_embeddings": getattr(cfg, "tie_embeddings", True),
        },
        "midi": midi or {},
        "source": source or {},
        "lm_head_alias": alias,
        "tensors": tensors,
    }
    hb = json.dumps(header, ensure_ascii=False).encode("utf-8")
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    with open(p, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", VERSION))
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for c in chunks:
            f.write(c)


def read_yuf(path):
    """Return (header dict, {name: ndarray}) with the tied head restored."""
    data = Path(path).read_bytes()
    if data[:4] != MAGIC:
        raise ValueError(f"{path}: bad magic")
    (ver,) = struct.unpack("<I", data[4:8])
    if ver != VERSION:
        raise ValueError(f"{path}: unsupported version {ver}")
    (hlen,) = struct.unpack("<Q", data[8:16])
    header = json.loads(data[16:16 + hlen].decode("utf-8"))
    blob = np.frombuffer(data, dtype="<f4", offset=16 + hlen)
    out = {}
    for t in header["tensors"]:
        out[t["name"]] = blob[t["offset"]:t["offset"] + t["count"]].reshape(t["shape"]).astype(np.float32)
    if header.get("lm_head_alias"):
        out["lm_head.weight"] = out[header["lm_head_alias"]]
    return header, out
