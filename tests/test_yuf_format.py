"""The .yuf container writer/reader (CPU): layout of
vulkan/scripts/export_checkpoint.py:47-146 (magic, version, header, data)."""

import json
import struct

import numpy as np

from yufmusicgen_b200 import config as C
from yufmusicgen_b200.weights import init_weights
from yufmusicgen_b200.yuf_format import read_yuf, write_yuf


def test_roundtrip_and_layout(tmp_path):
    cfg = C.ModelConfig(**C.TINY)
    w = init_weights(cfg, 0, "perturbed")
    p = tmp_path / "m.yuf"
    write_yuf(p, cfg, w)
    raw = p.read_bytes()
    assert raw[:4] == b"YUFM"
    assert struct.unpack("<I", raw[4:8])[0] == 1
    hlen = struct.unpack("<Q", raw[8:16])[0]
    header = json.loads(raw[16:16 + hlen])
    assert header["lm_head_alias"] == "token_embedding.weight"
    names = [t["name"] for t in header["tensors"]]
    assert names[0] == "token_embedding.weight"
    assert names[-2:] == ["final_norm.weight", "final_norm.bias"]
    assert "lm_head.weight" not in names
    assert header["model_config"]["d_model"] == cfg.d_model
    hdr, back = read_yuf(p)
    for k, v in w.items():
        np.testing.assert_array_equal(back[k], v)
    assert len(raw) == 16 + hlen + 4 * sum(t["count"] for t in header["tensors"])
