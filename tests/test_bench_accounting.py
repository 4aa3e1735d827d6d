"""The benchmark's algorithmic byte and FLOP accounting (no GPU): the figures
the roofline fractions in bench.py's JSON line are computed from.

* config 2: 7 N fp32 values per (b, t, h) (six inputs + y) plus the final
  N x N state per (b, h): 294.4 MB per step;
* config 4 decode step: every weight once and, per sequence, the recurrent
  state in and out (per layer prev [d], S [H, N, N], m [R]) -- about 2.95 MB
  of state per sequence on the 0.1B model, 112.75 M parameters in all.
"""

import bench
from yufmusicgen_b200 import config as C


def test_config2_algorithmic_bytes():
    assert bench.ALGO_BYTES == 8 * 2048 * 16 * 7 * 40 * 4 + 8 * 16 * 40 * 40 * 4
    assert abs(bench.ALGO_BYTES / 1e6 - 294.4) < 0.1


def test_decode_step_bytes_of_the_0p1b_model():
    cfg = C.ModelConfig(**C.BASE_0P1B)
    w32, state = bench.model_bytes_per_step(cfg, 4)
    w16, _ = bench.model_bytes_per_step(cfg, 2)
    assert abs(w32 / 4 / 1e6 - 112.75) < 0.2          # parameters (tied head counted once)
    assert w16 * 2 == w32
    per_layer_state = 2 * 4 * (640 + 16 * 40 * 40 + 128)
    assert state == 14 * per_layer_state + 4 * 20000   # + the logits row
    assert abs(14 * per_layer_state / 1e6 - 2.95) < 0.01
