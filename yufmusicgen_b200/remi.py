"""REMI token codec and MIDI files (C ABI ``yuf_remi_*`` / ``yuf_midi_*``), the
counterpart of the reference Vulkan client's ``RemiCodec`` and MIDI reader /
writer (vulkan/src/remi.rs, vulkan/src/midi.rs): generated token ids -> notes
-> a .mid file and back, without MidiTok.  Host code only (no GPU)."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from pathlib import Path

from . import _lib


@dataclass
class Note:
    start: int
    duration: int
    pitch: int
    velocity: int


@dataclass
class Track:
    program: int
    is_drum: bool = False
    name: str = ""
    notes: list[Note] = field(default_factory=list)


@dataclass
class Score:
    ticks_per_quarter: int
    tracks: list[Track] = field(default_factory=list)


class _NoteC(ctypes.Structure):
    _fields_ = [("start", ctypes.c_int32), ("duration", ctypes.c_int32), ("pitch", ctypes.c_int32),
                ("velocity", ctypes.c_int32)]


class _TrackC(ctypes.Structure):
    _fields_ = [("program", ctypes.c_int32), ("is_drum", ctypes.c_int32), ("name", ctypes.c_char_p),
                ("notes", ctypes.POINTER(_NoteC)), ("n_notes", ctypes.c_int64)]


def _tracks_c(score: Score):
    keep = []  # note arrays must outlive the call
    arr = (_TrackC * max(1, len(score.tracks)))()
    for i, t in enumerate(score.tracks):
        notes = (_NoteC * max(1, len(t.notes)))(*[_NoteC(n.start, n.duration, n.pitch, n.velocity)
                                                   for n in t.notes])
        keep.append(notes)
        arr[i] = _TrackC(int(t.program), 1 if t.is_drum else 0, (t.name or "").encode(),
                         ctypes.cast(notes, ctypes.POINTER(_NoteC)), len(t.notes))
    return arr, keep


def _gather(n_tracks, n_notes, programs, drums, notes, note_track, tpq, names=None):
    tracks = [Track(int(programs[i]), bool(drums[i]) if drums is not None else programs[i] == -1,
                    names[i] if names else "") for i in range(n_tracks)]
    for k in range(n_notes):
        n = notes[k]
        tracks[note_track[k]].notes.append(Note(n.start, n.duration, n.pitch, n.velocity))
    return Score(tpq, tracks)


class RemiCodec:
    """MidiTok 3.0 REMI as YufMusicGen configures it, over a vocabulary given
    as the list of token names by id (RemiCodec::new, remi.rs:35-62)."""

    def __init__(self, vocab: list[str]):
        self.vocab = list(vocab)
        arr = (ctypes.c_char_p * len(self.vocab))(*[v.encode() for v in self.vocab])
        h = ctypes.c_void_p()
        _lib.call("yuf_remi_create", arr, len(self.vocab), ctypes.byref(h))
        self._h = h

    def close(self):
        if self._h:
            _lib.call("yuf_remi_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def token_id(self, name: str) -> int | None:
        i = _lib.load().yuf_remi_token_id(self._h, name.encode())
        return None if i < 0 else int(i)

    def encode(self, score: Score) -> list[int]:
        """Score -> token ids (RemiCodec::encode, remi.rs:199-306)."""
        tracks, _keep = _tracks_c(score)
        n = ctypes.c_int64()
        _lib.call("yuf_remi_encode", self._h, score.ticks_per_quarter, tracks, len(score.tracks), None, 0,
                  ctypes.byref(n))
        out = (ctypes.c_int32 * max(1, n.value))()
        _lib.call("yuf_remi_encode", self._h, score.ticks_per_quarter, tracks, len(score.tracks), out,
                  n.value, ctypes.byref(n))
        return list(out[:n.value])

    def decode(self, ids) -> Score:
        """Token ids -> Score at 8 ticks per quarter (RemiCodec::decode, remi.rs:74-180)."""
        ids = [int(i) for i in ids]
        arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
        nt, nn = ctypes.c_int(), ctypes.c_int64()
        _lib.call("yuf_remi_decode", self._h, arr, len(ids), None, 0, ctypes.byref(nt), None, None, 0,
                  ctypes.byref(nn))
        progs = (ctypes.c_int32 * max(1, nt.value))()
        notes = (_NoteC * max(1, nn.value))()
        which = (ctypes.c_int32 * max(1, nn.value))()
        _lib.call("yuf_remi_decode", self._h, arr, len(ids), progs, nt.value, ctypes.byref(nt), notes, which,
                  nn.value, ctypes.byref(nn))
        return _gather(nt.value, nn.value, progs, None, notes, which, 8)


def render_midi(score: Score) -> bytes:
    """Score -> format-1 Standard MIDI File bytes (render_midi, midi.rs:351-402)."""
    tracks, _keep = _tracks_c(score)
    n = ctypes.c_int64()
    _lib.call("yuf_midi_render", score.ticks_per_quarter, tracks, len(score.tracks), None, 0, ctypes.byref(n))
    out = (ctypes.c_uint8 * n.value)()
    _lib.call("yuf_midi_render", score.ticks_per_quarter, tracks, len(score.tracks), out, n.value,
              ctypes.byref(n))
    return bytes(out)


def parse_midi(data: bytes) -> Score:
    """Standard MIDI File bytes -> Score (parse_midi, midi.rs:64-281)."""
    buf = (ctypes.c_uint8 * len(data)).from_buffer_copy(data)
    tpq, nt, nn = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    _lib.call("yuf_midi_parse", buf, len(data), ctypes.byref(tpq), None, None, 0, ctypes.byref(nt), None, None,
              0, ctypes.byref(nn))
    progs = (ctypes.c_int32 * max(1, nt.value))()
    drums = (ctypes.c_int32 * max(1, nt.value))()
    notes = (_NoteC * max(1, nn.value))()
    which = (ctypes.c_int32 * max(1, nn.value))()
    _lib.call("yuf_midi_parse", buf, len(data), ctypes.byref(tpq), progs, drums, nt.value, ctypes.byref(nt),
              notes, which, nn.value, ctypes.byref(nn))
    return _gather(nt.value, nn.value, progs, drums, notes, which, tpq.value)


def midi_ids(tokens, vocab_size: int, offset: int | None = None) -> list[int]:
    """Model token ids -> the codec's raw MidiTok ids: the tokens in
    [MIDI_OFFSET, vocab_size) shifted down by MIDI_OFFSET, other ids (text
    bytes, specials) dropped -- what the reference does with a generated
    sequence before decoding it (vulkan/src/generation.rs:218-232)."""
    from .config import MIDI_OFFSET

    off = MIDI_OFFSET if offset is None else offset
    return [int(t) - off for t in tokens if off <= int(t) < vocab_size]


def write_midi(path, score: Score) -> None:
    Path(path).write_bytes(render_midi(score))


def read_midi(path) -> Score:
    return parse_midi(Path(path).read_bytes())
