"""Seeded synthetic weights with the reference's parameter names and shapes.

There are no trained checkpoints on this machine, so every workload runs on
random-init weights.  The names and shapes are those of the reference
``YufMusicGen.state_dict()`` (``yufmusicgen/model.py:40-392``), so a dict
produced here loads into the reference model with ``load_state_dict`` and a
reference checkpoint's ``state_dict`` loads into the engine unchanged.

Init recipe (``recipe="baseline"``):

* every matrix (embedding, ``nn.Linear`` weights, the low-rank ``w1/w2``,
  ``a1/a2``, ``g1/g2``) ~ N(0, 0.02);
* ``w0 = a0 = 0`` and ``rosa.decay = 0`` (the "decay/a biases zero" of the
  benchmark configs);
* ``mix_*``, ``k_k``, ``k_a`` = the reference constructor's values for
  ``layer_id=0`` (``yufmusicgen/model.py:50-57, 72-73``; ``YufBlock`` never
  passes a layer id) plus N(0, 0.02);
* ``householder`` ~ N(0, 1) (``yufmusicgen/model.py:213``);
* LayerNorm weight 1, bias 0; ROSA projection biases 0.

``recipe="perturbed"`` additionally draws every LayerNorm affine, the ROSA
biases, ``w0``, ``a0`` and ``decay`` at random so parity tests exercise every
parameter.  The generator is numpy's PCG64 with a fixed seed, which gives the
same bits on every machine with the same numpy.
"""

from __future__ import annotations

import numpy as np

from .config import ModelConfig


def _ln(rng, d, perturbed):
    if perturbed:
        return (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32), (
            0.1 * rng.standard_normal(d)
        ).astype(np.float32)
    return np.ones(d, np.float32), np.zeros(d, np.float32)


def init_weights(cfg: ModelConfig, seed: int, recipe: str = "baseline") -> dict[str, np.ndarray]:
    if recipe not in ("baseline", "perturbed"):
        raise ValueError(f"unknown init recipe {recipe!r}")
    cfg.validate()
    pert = recipe == "perturbed"
    rng = np.random.default_rng(seed)
    d, lr, R, V, F = cfg.d_model, cfg.low_rank, cfg.rosa_size, cfg.vocab_size, cfg.ffn_hidden

    def mat(*shape, std=0.02):
        return (std * rng.standard_normal(shape)).astype(np.float32)

    out: dict[str, np.ndarray] = {}
    out["token_embedding.weight"] = mat(V, d)
    ramp = np.linspace(0.0, 1.0, d, dtype=np.float32)
    ratio = 1.0  # layer_id = 0 in every block (yufmusicgen/model.py:349)
    mix_pow = dict(r=0.2, w=0.9, k=0.7, v=0.7, a=0.9, g=0.2)
    for i in range(cfg.n_layers):
        p = f"blocks.{i}."
        out[p + "norm_time.weight"], out[p + "norm_time.bias"] = _ln(rng, d, pert)
        tm = p + "time_mix."
        for name, pw in mix_pow.items():
            base = 1.0 - np.power(ramp, pw * ratio)
            out[tm + f"mix_{name}"] = (base + 0.02 * rng.standard_normal(d)).astype(np.float32)
        out[tm + "w0"] = (0.5 * rng.standard_normal(d)).astype(np.float32) if pert else np.zeros(d, np.float32)
        out[tm + "w1"] = mat(d, lr)
        out[tm + "w2"] = mat(lr, d)
        out[tm + "a0"] = (0.5 * rng.standard_normal(d)).astype(np.float32) if pert else np.zeros(d, np.float32)
        out[tm + "a1"] = mat(d, lr)
        out[tm + "a2"] = mat(lr, d)
        out[tm + "g1"] = mat(d, lr)
        out[tm + "g2"] = mat(lr, d)
        out[tm + "k_k"] = (0.71 + 0.02 * rng.standard_normal(d)).astype(np.float32)
        out[tm + "k_a"] = (1.02 + 0.02 * rng.standard_normal(d)).astype(np.float32)
        out[tm + "receptance.weight"] = mat(d, d)
        out[tm + "key.weight"] = mat(d, d)
        out[tm + "value.weight"] = mat(d, d)
        out[tm + "output.weight"] = mat(d, d)
        out[tm + "out_norm.weight"], out[tm + "out_norm.bias"] = _ln(rng, d, pert)
        out[p + "norm_rosa.weight"], out[p + "norm_rosa.bias"] = _ln(rng, d, pert)
        ro = p + "rosa."
        out[ro + "householder"] = rng.standard_normal(R).astype(np.float32)
        out[ro + "decay"] = rng.standard_normal(R).astype(np.float32) if pert else np.zeros(R, np.float32)
        for proj in ("input", "write_gate", "read_gate"):
            out[ro + proj + ".weight"] = mat(R, d)
            out[ro + proj + ".bias"] = mat(R, std=0.1) if pert else np.zeros(R, np.float32)
        out[ro + "output.weight"] = mat(d, R)
        out[p + "norm_ffn.weight"], out[p + "norm_ffn.bias"] = _ln(rng, d, pert)
        out[p + "ffn_in.weight"] = mat(F, d)
        out[p + "ffn_gate.weight"] = mat(F, d)
        out[p + "ffn_out.weight"] = mat(d, F)
    out["final_norm.weight"], out["final_norm.bias"] = _ln(rng, d, pert)
    if cfg.tie_embeddings:
        out["lm_head.weight"] = out["token_embedding.weight"]
    else:
        out["lm_head.weight"] = mat(V, d)
    return out
