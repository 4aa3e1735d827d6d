"""Model configuration for the B200 engine.

Mirrors ``ModelConfig`` in ``yufmusicgen/config.py:74-93`` of the reference:
the same field names, defaults and validation rules, so a reference
checkpoint's ``model_config`` dict loads unchanged (unknown keys are ignored,
as in ``dataclass_from_dict``, ``yufmusicgen/config.py:115-119``).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any

# Token layout of the reference tokenizer (yufmusicgen/tokenizer.py:10-16).
PAD, BOS, EOS, SEP = 0, 1, 2, 3
BYTE_OFFSET = 4
MIDI_OFFSET = 260


@dataclass
class ModelConfig:
    vocab_size: int = 673
    d_model: int = 640
    n_layers: int = 14
    n_heads: int = 16
    head_size: int = 40
    rosa_size: int = 128
    dropout: float = 0.0
    tie_embeddings: bool = True
    use_cuda_kernel: bool = True
    use_rosa_scan: bool = True

    def validate(self) -> None:
        # yufmusicgen/config.py:87-93
        if self.d_model != self.n_heads * self.head_size:
            raise ValueError("d_model must equal n_heads * head_size")
        if self.d_model < 32 or self.n_layers < 1:
            raise ValueError("model is too small to be useful")
        if self.head_size > 1024:
            raise ValueError("head_size must fit within one CUDA thread block")

    @property
    def low_rank(self) -> int:
        """Width of the w/a/g low-rank projections.

        ``max(32, int(round(2.5 * sqrt(d) / 32) * 32))`` exactly as
        ``yufmusicgen/model.py:59`` computes it: Python's ``round`` is
        round-half-to-even, so d=1024 gives 64 (the Rust exporter's
        ``checkpoint.rs:27-30`` rounds half away from zero and would give 96;
        the Python rule is the one the trained weights follow).
        """
        return max(32, int(round(2.5 * (self.d_model ** 0.5) / 32) * 32))

    @property
    def ffn_hidden(self) -> int:
        return 4 * self.d_model  # yufmusicgen/model.py:353

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict[str, Any]) -> "ModelConfig":
        fields = cls.__dataclass_fields__
        return cls(**{k: v for k, v in values.items() if k in fields})


# Named configurations of the benchmark workloads (model part only).
TINY = dict(vocab_size=512, d_model=128, n_layers=2, n_heads=4, head_size=32, rosa_size=32)
BASE_0P1B = dict(vocab_size=20000, d_model=640, n_layers=14, n_heads=16, head_size=40, rosa_size=128)
LONG_1K = dict(vocab_size=20000, d_model=1024, n_layers=24, n_heads=16, head_size=64, rosa_size=256)
# The configuration of the reference's own state test (tests/test_model_state.py:11-18).
STATE_TEST = dict(vocab_size=300, d_model=32, n_layers=2, n_heads=2, head_size=16, rosa_size=12)
