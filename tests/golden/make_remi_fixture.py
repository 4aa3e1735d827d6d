"""Write the REMI vocabulary fixture from the reference tree.

The reference's REMI codec (vulkan/src/remi.rs) works on MidiTok 3.0's
vocabulary for the project's codec configuration; its tests load that
vocabulary from vulkan/testdata/vocab.json (vulkan/tests/remi_tests.rs:9-13).
This script writes the same list as tests/golden/remi_vocab.json, so the GPU
box and this repository's tests need no reference tree:

    YUF_REFERENCE=/path/to/YufMusicGen python tests/golden/make_remi_fixture.py
"""

import json
import os
import sys
from pathlib import Path

ref = os.environ.get("YUF_REFERENCE")
if not ref:
    raise SystemExit("set YUF_REFERENCE to the reference source tree")
vocab = json.loads((Path(ref) / "vulkan" / "testdata" / "vocab.json").read_text())
if not (isinstance(vocab, list) and all(isinstance(t, str) for t in vocab)):
    sys.exit("unexpected vocabulary format")
out = Path(__file__).resolve().parent / "remi_vocab.json"
out.write_text(json.dumps(vocab, indent=0) + "\n")
print(f"wrote {out} ({len(vocab)} tokens)")
