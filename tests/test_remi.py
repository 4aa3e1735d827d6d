"""REMI codec and MIDI file I/O (C ABI yuf_remi_* / yuf_midi_*; CPU only).

Known answers from the reference's own codec tests
(vulkan/tests/remi_tests.rs:47-200, captured there from MidiTok 3.0 through
yufmusicgen + Python) over its vocabulary fixture
(tests/golden/remi_vocab.json, written by tests/golden/make_remi_fixture.py)."""

import json
from pathlib import Path

import pytest

from yufmusicgen_b200.remi import Note, RemiCodec, Score, Track, parse_midi, read_midi, render_midi, write_midi

VOCAB = json.loads((Path(__file__).resolve().parent / "golden" / "remi_vocab.json").read_text())
TOKENS = [4, 190, 284, 44, 117, 127, 192, 324, 56, 115, 129, 194, 284, 48, 118, 129, 198, 284, 51, 113, 126]


@pytest.fixture(scope="module")
def codec():
    c = RemiCodec(VOCAB)
    yield c
    c.close()


def two_track_score():
    return Score(480, [
        Track(0, False, "Piano", [Note(0, 120, 60, 96), Note(240, 240, 64, 100), Note(480, 60, 67, 80)]),
        Track(40, False, "Violin", [Note(120, 240, 72, 88)]),
    ])


def test_encode_matches_miditok_reference(codec):
    assert codec.encode(two_track_score()) == TOKENS


def test_decode_matches_miditok_reference(codec):
    s = codec.decode(TOKENS)
    assert s.ticks_per_quarter == 8 and len(s.tracks) == 2
    assert s.tracks[0].program == 0
    assert s.tracks[0].notes == [Note(0, 2, 60, 95), Note(4, 4, 64, 99), Note(8, 1, 67, 79)]
    assert s.tracks[1].program == 40
    assert s.tracks[1].notes == [Note(2, 4, 72, 87)]


def test_duration_quantization_matches_miditok(codec):
    names = ["Bar_None", "Position_0", "Program_0", "Pitch_60", "Velocity_99", "Duration_0.2.8",
             "Position_12", "Program_0", "Pitch_61", "Velocity_99", "Duration_0.3.8",
             "Position_23", "Program_0", "Pitch_62", "Velocity_99", "Duration_0.5.8",
             "Bar_None", "Position_3", "Program_0", "Pitch_63", "Velocity_99", "Duration_1.2.8",
             "Position_15", "Program_0", "Pitch_64", "Velocity_99", "Duration_1.7.8",
             "Position_26", "Program_0", "Pitch_65", "Velocity_99", "Duration_4.1.4"]
    want = [codec.token_id(n) for n in names]
    assert None not in want
    score = Score(480, [Track(0, False, "", [
        Note(0, 90, 60, 100), Note(700, 150, 61, 100), Note(1400, 300, 62, 100),
        Note(2100, 620, 63, 100), Note(2800, 900, 64, 100), Note(3500, 2000, 65, 100)])])
    assert codec.encode(score) == want


def test_decode_encode_roundtrip_is_stable(codec):
    tokens = codec.encode(two_track_score())
    assert codec.encode(codec.decode(tokens)) == tokens


def _notes(score):
    return sorted((n.start, n.duration, n.pitch, n.velocity) for t in score.tracks for n in t.notes)


def test_midi_file_roundtrip():
    parsed = parse_midi(render_midi(two_track_score()))
    assert parsed.ticks_per_quarter == 480 and len(parsed.tracks) == 2
    assert sorted((n.start, n.duration, n.pitch, n.velocity) for n in parsed.tracks[0].notes) == [
        (0, 120, 60, 96), (240, 240, 64, 100), (480, 60, 67, 80)]
    assert parsed.tracks[1].program == 40


def test_decode_midi_render_parse_roundtrip(codec):
    parsed = parse_midi(render_midi(codec.decode(TOKENS)))
    assert _notes(parsed) == [(0, 2, 60, 95), (2, 4, 72, 87), (4, 4, 64, 99), (8, 1, 67, 79)]


def test_write_read_midi_file(tmp_path):
    path = tmp_path / "roundtrip.mid"
    write_midi(path, two_track_score())
    loaded = read_midi(path)
    assert len(loaded.tracks) == 2 and len(loaded.tracks[0].notes) == 3


def test_overlapping_notes_keep_their_times():
    """Chords and overlapping notes survive render -> parse unchanged (the
    reference writer serialises a track's notes and would shift them)."""
    s = Score(96, [Track(5, False, "", [Note(0, 96, 60, 90), Note(0, 96, 64, 80), Note(48, 96, 67, 70)]),
                   Track(0, True, "", [Note(0, 24, 36, 100), Note(24, 24, 38, 100)])])
    p = parse_midi(render_midi(s))
    assert _notes(p) == _notes(s)
    assert [t.is_drum for t in p.tracks] == [False, True] and p.tracks[0].program == 5


def test_errors_are_reported(codec):
    from yufmusicgen_b200._lib import YufError

    with pytest.raises(YufError, match="not a MIDI file"):
        parse_midi(b"RIFF" + bytes(20))
    with pytest.raises(YufError, match="ticks-per-quarter"):
        codec.encode(Score(0, []))
    # Program 200 has no token in the vocabulary
    with pytest.raises(YufError, match="not in the vocabulary"):
        codec.encode(Score(8, [Track(200, False, "", [Note(0, 8, 60, 100)])]))
    assert codec.decode([]).tracks == [] and codec.decode([99999, -3, 4]).tracks == []


def test_generated_tokens_to_midi_ids(codec):
    """Model ids -> codec ids as the reference's generation loop does: only the
    MIDI range, shifted by MIDI_OFFSET (260); then decode."""
    from yufmusicgen_b200.config import MIDI_OFFSET
    from yufmusicgen_b200.remi import midi_ids

    model_tokens = [1, 4 + 65, *(t + MIDI_OFFSET for t in TOKENS), 2]  # BOS, a byte, the music, EOS
    assert midi_ids(model_tokens, vocab_size=MIDI_OFFSET + len(VOCAB)) == TOKENS
    assert len(codec.decode(midi_ids(model_tokens, MIDI_OFFSET + len(VOCAB))).tracks) == 2


def test_codec_from_a_yuf_export(tmp_path):
    """The exporter stores the MIDI vocabulary in the .yuf header
    (vulkan/scripts/export_checkpoint.py:117-123); the codec reads it from there."""
    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.weights import init_weights
    from yufmusicgen_b200.yuf_format import read_yuf, write_yuf

    cfg = C.ModelConfig(**C.TINY)
    path = tmp_path / "tiny.yuf"
    write_yuf(path, cfg, init_weights(cfg, 0, "perturbed"),
              midi={"tokenization": "REMI", "midi_offset": 260, "midi_vocab_size": len(VOCAB), "vocab": VOCAB})
    header, _ = read_yuf(path)
    c = RemiCodec(header["midi"]["vocab"])
    assert c.encode(two_track_score()) == TOKENS
    c.close()
