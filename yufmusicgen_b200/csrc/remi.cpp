// REMI token codec and Standard MIDI File I/O (host code; C ABI in
// include/yufb200.h).
//
// The generation loop emits MidiTok ids; this file turns them into notes and a
// .mid file and back, as the reference's Vulkan client does in Rust
// (vulkan/src/remi.rs, vulkan/src/midi.rs) for MidiTok 3.0's REMI in the
// project's configuration: no BPE, no tempo / time-signature / rest / chord
// tokens, one token stream in which every note carries its Program token.
//
// Token grammar (one bar = 32 positions of 1 tick at 8 ticks per quarter):
//   Bar_None                      next bar
//   Position_<p>                  tick = bar start + p
//   Program_<n>                   program of the following notes (-1 = drums)
//   Pitch_<k> | PitchDrum_<k>     a note, followed by Velocity_<v> and
//   Velocity_<v>, Duration_<b>.<p>.<r>   a duration of (b r + p) * 8 / r ticks

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/yufb200.h"

namespace yuf {
void set_error(const char* fmt, ...);
}  // namespace yuf

using yuf::set_error;

namespace {

constexpr int kTpq = 8;          // ticks per quarter of the token grid
constexpr int kTicksPerBar = 32;  // 4/4
constexpr int kPitchMin = 21, kPitchMax = 109;
constexpr int kDrumPitchMin = 27, kDrumPitchMax = 88;

// Index of the value of a sorted list nearest to v; a tie goes to the larger
// value (MidiTok's np.searchsorted(side="left") based snapping).
size_t nearest_tie_up(const std::vector<int>& sorted, int v) {
  const size_t hi = std::lower_bound(sorted.begin(), sorted.end(), v) - sorted.begin();
  if (hi == sorted.size()) return hi - 1;
  if (hi > 0 && v - sorted[hi - 1] < sorted[hi] - v) return hi - 1;
  return hi;
}

int round_half_up(double x) { return (int)std::floor(x + 0.5); }

// "<beat>.<pos>.<res>" -> ticks at kTpq, or -1 when malformed.
int duration_ticks(const std::string& value) {
  int beat = 0, pos = 0, res = 0;
  char tail = 0;
  if (std::sscanf(value.c_str(), "%d.%d.%d%c", &beat, &pos, &res, &tail) != 3 || res <= 0) return -1;
  return (beat * res + pos) * kTpq / res;
}

bool parse_int(const std::string& s, int* out) {
  if (s.empty()) return false;
  char* end = nullptr;
  const long v = std::strtol(s.c_str(), &end, 10);
  if (*end != 0) return false;
  *out = (int)v;
  return true;
}

struct Note {
  int start, duration, pitch, velocity;
};

}  // namespace

struct yuf_remi {
  std::vector<std::string> vocab;
  std::unordered_map<std::string, int32_t> ids;
  std::vector<int> dur_ticks;            // distinct Duration lengths, ascending
  std::vector<std::string> dur_value;    // the first token value with each length
  std::vector<int> velocities;           // 3, 7, ..., 127

  // split "Kind_value"; false when there is no '_'
  bool split(int32_t id, std::string* kind, std::string* value) const {
    if (id < 0 || (size_t)id >= vocab.size()) return false;
    const std::string& name = vocab[id];
    const size_t u = name.find('_');
    if (u == std::string::npos) return false;
    *kind = name.substr(0, u);
    *value = name.substr(u + 1);
    return true;
  }
};

extern "C" {

yuf_status_t yuf_remi_create(const char* const* vocab, int n_vocab, yuf_remi** out) {
  if (!vocab || n_vocab <= 0 || !out) {
    set_error("remi: need a non-empty vocabulary and an output handle");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  auto* c = new yuf_remi();
  std::vector<std::pair<int, std::string>> durs;
  for (int i = 0; i < n_vocab; ++i) {
    if (!vocab[i]) {
      delete c;
      set_error("remi: vocabulary entry %d is NULL", i);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    c->vocab.emplace_back(vocab[i]);
    c->ids.emplace(c->vocab.back(), i);  // the first id of a repeated name wins
    const std::string& name = c->vocab.back();
    if (name.rfind("Duration_", 0) == 0) {
      const int t = duration_ticks(name.substr(9));
      if (t < 0) {
        delete c;
        set_error("remi: malformed duration token %s", name.c_str());
        return YUF_ERR_INVALID_ARGUMENT;
      }
      durs.emplace_back(t, name.substr(9));
    }
  }
  std::stable_sort(durs.begin(), durs.end(),
                   [](const auto& a, const auto& b) { return a.first < b.first; });
  for (const auto& d : durs)
    if (c->dur_ticks.empty() || c->dur_ticks.back() != d.first) {
      c->dur_ticks.push_back(d.first);
      c->dur_value.push_back(d.second);
    }
  for (int v = 3; v <= 127; v += 4) c->velocities.push_back(v);
  *out = c;
  return YUF_OK;
}

yuf_status_t yuf_remi_destroy(yuf_remi* codec) {
  delete codec;
  return YUF_OK;
}

int32_t yuf_remi_token_id(const yuf_remi* codec, const char* name) {
  if (!codec || !name) return -1;
  auto it = codec->ids.find(name);
  return it == codec->ids.end() ? -1 : it->second;
}

yuf_status_t yuf_remi_encode(const yuf_remi* codec, int ticks_per_quarter,
                             const yuf_track_desc* tracks, int n_tracks, int32_t* ids,
                             int64_t capacity, int64_t* n_ids) {
  if (!codec || !n_ids || n_tracks < 0 || (n_tracks > 0 && !tracks)) {
    set_error("remi encode: null codec, tracks or n_ids");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (ticks_per_quarter <= 0) {
    set_error("remi encode: the score has no ticks-per-quarter division");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (codec->dur_ticks.empty()) {
    set_error("remi encode: the vocabulary has no Duration tokens");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  const double scale = (double)kTpq / ticks_per_quarter;
  // tracks sharing (program, drum) become one, in order of first appearance
  struct Group {
    int program;
    bool drum;
    std::vector<Note> notes;
  };
  std::vector<Group> groups;
  for (int t = 0; t < n_tracks; ++t) {
    const yuf_track_desc& tr = tracks[t];
    if (tr.n_notes < 0 || (tr.n_notes > 0 && !tr.notes)) {
      set_error("remi encode: track %d has no note array", t);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    const bool drum = tr.is_drum != 0;
    auto g = std::find_if(groups.begin(), groups.end(),
                          [&](const Group& x) { return x.program == tr.program && x.drum == drum; });
    if (g == groups.end()) g = groups.insert(groups.end(), Group{tr.program, drum, {}});
    for (int64_t i = 0; i < tr.n_notes; ++i) {
      const yuf_note& n = tr.notes[i];
      if (n.start < 0 || n.duration < 0) {
        set_error("remi encode: note %lld of track %d has a negative time", (long long)i, t);
        return YUF_ERR_INVALID_ARGUMENT;
      }
      g->notes.push_back({n.start, n.duration, n.pitch, n.velocity});
    }
  }
  struct Event {
    int time;
    std::string name;
  };
  std::vector<Event> events;
  for (Group& g : groups) {
    std::vector<Note> notes;
    const int lo = g.drum ? kDrumPitchMin : kPitchMin, hi = g.drum ? kDrumPitchMax : kPitchMax;
    for (const Note& n : g.notes) {
      if (n.pitch < lo || n.pitch > hi) continue;
      notes.push_back({round_half_up(n.start * scale), std::max(1, round_half_up(n.duration * scale)),
                       n.pitch, codec->velocities[nearest_tie_up(codec->velocities, n.velocity)]});
    }
    std::stable_sort(notes.begin(), notes.end(), [](const Note& a, const Note& b) {
      if (a.start != b.start) return a.start < b.start;
      if (a.duration != b.duration) return a.duration < b.duration;
      return a.pitch < b.pitch;
    });
    const std::string prog = "Program_" + std::to_string(g.program);
    const std::string pitch_kind = g.drum ? "PitchDrum_" : "Pitch_";
    for (const Note& n : notes) {
      events.push_back({n.start, prog});
      events.push_back({n.start, pitch_kind + std::to_string(n.pitch)});
      events.push_back({n.start, "Velocity_" + std::to_string(n.velocity)});
      events.push_back({n.start, "Duration_" + codec->dur_value[nearest_tie_up(codec->dur_ticks, n.duration)]});
    }
  }
  std::stable_sort(events.begin(), events.end(), [](const Event& a, const Event& b) { return a.time < b.time; });
  // time tokens: Bar_None for every bar boundary crossed, Position_<p> at each new time
  std::vector<int32_t> out;
  int bar = -1, bar_tick = 0, prev = -1;
  auto emit = [&](const std::string& name) -> bool {
    const int32_t id = yuf_remi_token_id(codec, name.c_str());
    if (id < 0) {
      set_error("remi encode: token %s is not in the vocabulary", name.c_str());
      return false;
    }
    out.push_back(id);
    return true;
  };
  for (const Event& e : events) {
    if (e.time != prev) {
      for (int b = e.time / kTicksPerBar - bar; b > 0; --b) {
        ++bar;
        bar_tick = bar * kTicksPerBar;
        if (!emit("Bar_None")) return YUF_ERR_INVALID_ARGUMENT;
      }
      if (!emit("Position_" + std::to_string(e.time - bar_tick))) return YUF_ERR_INVALID_ARGUMENT;
      prev = e.time;
    }
    if (!emit(e.name)) return YUF_ERR_INVALID_ARGUMENT;
  }
  *n_ids = (int64_t)out.size();
  if (ids) {
    if (capacity < (int64_t)out.size()) {
      set_error("remi encode: %lld ids do not fit in %lld", (long long)out.size(), (long long)capacity);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    std::copy(out.begin(), out.end(), ids);
  }
  return YUF_OK;
}

yuf_status_t yuf_remi_decode(const yuf_remi* codec, const int32_t* ids, int64_t n_ids,
                             int32_t* track_programs, int max_tracks, int* n_tracks,
                             yuf_note* notes, int32_t* note_track, int64_t max_notes,
                             int64_t* n_notes) {
  if (!codec || !n_tracks || !n_notes || n_ids < 0 || (n_ids > 0 && !ids)) {
    set_error("remi decode: null codec, ids or counts");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  std::vector<int32_t> programs;
  std::vector<std::pair<int32_t, yuf_note>> out;  // (track index, note)
  int bar = -1, bar_tick = 0, tick = 0, program = 0;
  std::string kind, value, k2, v2, k3, v3;
  for (int64_t i = 0; i < n_ids; ++i) {
    if (!codec->split(ids[i], &kind, &value)) continue;
    int x = 0;
    if (kind == "Bar") {
      ++bar;
      bar_tick = bar * kTicksPerBar;
      tick = bar_tick;
    } else if (kind == "Position") {
      if (bar == -1) bar = 0;
      tick = bar_tick + (parse_int(value, &x) ? x : 0);
    } else if (kind == "Program") {
      program = parse_int(value, &x) ? x : 0;
    } else if (kind == "Pitch" || kind == "PitchDrum") {
      if (!parse_int(value, &x) || x < kPitchMin || x > kPitchMax) continue;
      int vel = -1, dur = -1, y = 0;
      if (i + 1 < n_ids && codec->split(ids[i + 1], &k2, &v2) && k2 == "Velocity" && parse_int(v2, &y) &&
          y >= 0 && y <= 255)
        vel = y;
      if (i + 2 < n_ids && codec->split(ids[i + 2], &k3, &v3) && k3 == "Duration") dur = duration_ticks(v3);
      if (vel < 0 || dur < 0) continue;
      auto it = std::find(programs.begin(), programs.end(), program);
      const int32_t ti = (int32_t)(it - programs.begin());
      if (it == programs.end()) programs.push_back(program);
      out.push_back({ti, yuf_note{tick, dur, x, vel}});
    }
  }
  *n_tracks = (int)programs.size();
  *n_notes = (int64_t)out.size();
  if (track_programs) {
    if (max_tracks < (int)programs.size()) {
      set_error("remi decode: %zu tracks do not fit in %d", programs.size(), max_tracks);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    std::copy(programs.begin(), programs.end(), track_programs);
  }
  if (notes) {
    if (max_notes < (int64_t)out.size() || !note_track) {
      set_error("remi decode: %zu notes do not fit in %lld (or note_track is NULL)", out.size(),
                (long long)max_notes);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    for (size_t i = 0; i < out.size(); ++i) {
      notes[i] = out[i].second;
      note_track[i] = out[i].first;
    }
  }
  return YUF_OK;
}

// ---- Standard MIDI File ----------------------------------------------------

namespace {

void put_u32(std::vector<uint8_t>& o, uint32_t v) {
  for (int s = 24; s >= 0; s -= 8) o.push_back((uint8_t)(v >> s));
}
void put_u16(std::vector<uint8_t>& o, uint16_t v) {
  o.push_back((uint8_t)(v >> 8));
  o.push_back((uint8_t)v);
}
void put_varlen(std::vector<uint8_t>& o, uint32_t v) {
  uint8_t buf[5];
  int n = 0;
  buf[n++] = (uint8_t)(v & 0x7F);
  while (v >>= 7) buf[n++] = (uint8_t)(0x80 | (v & 0x7F));
  while (n) o.push_back(buf[--n]);
}

struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  uint8_t u8() {
    if (pos >= n) { ok = false; return 0; }
    return p[pos++];
  }
  uint32_t u32() { uint32_t v = 0; for (int i = 0; i < 4; ++i) v = (v << 8) | u8(); return v; }
  uint16_t u16() { uint16_t v = (uint16_t)(u8() << 8); return (uint16_t)(v | u8()); }
  uint32_t varlen() {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const uint8_t b = u8();
      v = (v << 7) | (b & 0x7F);
      if (!(b & 0x80)) return v;
    }
    ok = false;  // more than four bytes
    return v;
  }
  void skip(size_t k) {
    if (k > n - pos) { ok = false; pos = n; return; }
    pos += k;
  }
};

}  // namespace

yuf_status_t yuf_midi_render(int ticks_per_quarter, const yuf_track_desc* tracks, int n_tracks,
                             uint8_t* out, int64_t capacity, int64_t* n_bytes) {
  if (!n_bytes || n_tracks < 0 || n_tracks > 65535 || (n_tracks > 0 && !tracks) ||
      ticks_per_quarter <= 0 || ticks_per_quarter > 0x7FFF) {
    set_error("midi render: need n_bytes, 0..65535 tracks and a division in 1..32767");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  std::vector<uint8_t> f = {'M', 'T', 'h', 'd'};
  put_u32(f, 6);
  put_u16(f, 1);  // format 1
  put_u16(f, (uint16_t)n_tracks);
  put_u16(f, (uint16_t)ticks_per_quarter);
  for (int t = 0; t < n_tracks; ++t) {
    const yuf_track_desc& tr = tracks[t];
    if (tr.n_notes < 0 || (tr.n_notes > 0 && !tr.notes)) {
      set_error("midi render: track %d has no note array", t);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    const uint8_t ch = tr.is_drum ? 9 : (uint8_t)(((tr.program % 16) + 16) % 16);
    std::vector<uint8_t> b;
    std::string name = tr.name ? tr.name : "";
    if (name.empty()) name = tr.is_drum ? "Drums" : "Program " + std::to_string(tr.program);
    put_varlen(b, 0);
    b.push_back(0xFF);
    b.push_back(0x03);
    put_varlen(b, (uint32_t)name.size());
    b.insert(b.end(), name.begin(), name.end());
    put_varlen(b, 0);
    b.push_back((uint8_t)(0xC0 | ch));
    b.push_back(tr.is_drum ? 0 : (uint8_t)(tr.program & 0x7F));
    // note-on / note-off events in time order; at equal times note-offs first
    struct Ev {
      int64_t tick;
      int on;
      int pitch, velocity;
    };
    std::vector<Ev> ev;
    for (int64_t i = 0; i < tr.n_notes; ++i) {
      const yuf_note& n = tr.notes[i];
      if (n.start < 0 || n.pitch < 0 || n.pitch > 127 || n.velocity < 1 || n.velocity > 127) {
        set_error("midi render: note %lld of track %d is out of range", (long long)i, t);
        return YUF_ERR_INVALID_ARGUMENT;
      }
      ev.push_back({n.start, 1, n.pitch, n.velocity});
      ev.push_back({(int64_t)n.start + std::max(1, n.duration), 0, n.pitch, 0});
    }
    std::stable_sort(ev.begin(), ev.end(), [](const Ev& a, const Ev& b) {
      if (a.tick != b.tick) return a.tick < b.tick;
      if (a.on != b.on) return a.on < b.on;
      return a.pitch < b.pitch;
    });
    int64_t last = 0;
    for (const Ev& e : ev) {
      put_varlen(b, (uint32_t)(e.tick - last));
      last = e.tick;
      b.push_back((uint8_t)((e.on ? 0x90 : 0x80) | ch));
      b.push_back((uint8_t)e.pitch);
      b.push_back((uint8_t)e.velocity);
    }
    put_varlen(b, 0);
    b.push_back(0xFF);
    b.push_back(0x2F);
    b.push_back(0x00);
    f.insert(f.end(), {'M', 'T', 'r', 'k'});
    put_u32(f, (uint32_t)b.size());
    f.insert(f.end(), b.begin(), b.end());
  }
  *n_bytes = (int64_t)f.size();
  if (out) {
    if (capacity < (int64_t)f.size()) {
      set_error("midi render: %zu bytes do not fit in %lld", f.size(), (long long)capacity);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    std::memcpy(out, f.data(), f.size());
  }
  return YUF_OK;
}

yuf_status_t yuf_midi_parse(const uint8_t* bytes, int64_t n_bytes, int* ticks_per_quarter,
                            int32_t* track_programs, int32_t* track_is_drum, int max_tracks,
                            int* n_tracks, yuf_note* notes, int32_t* note_track,
                            int64_t max_notes, int64_t* n_notes) {
  if (!bytes || n_bytes < 14 || !ticks_per_quarter || !n_tracks || !n_notes) {
    set_error("midi parse: need the file bytes (at least a header) and the count outputs");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  Reader r{bytes, (size_t)n_bytes};
  if (std::memcmp(bytes, "MThd", 4) != 0) {
    set_error("midi parse: not a MIDI file (no MThd chunk)");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  r.skip(4);
  const uint32_t hlen = r.u32();
  r.u16();  // format
  const uint16_t ntrk = r.u16();
  const uint16_t division = r.u16();
  if (!r.ok || hlen < 6 || (division & 0x8000)) {
    set_error("midi parse: bad header or SMPTE timing (not supported)");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  r.skip(hlen - 6);
  struct Track {
    int program, drum;
    std::vector<yuf_note> notes;
  };
  std::vector<Track> tracks;
  for (int t = 0; t < ntrk && r.ok; ++t) {
    const size_t at = r.pos;
    if (r.n - r.pos < 8 || std::memcmp(bytes + at, "MTrk", 4) != 0) {
      set_error("midi parse: expected an MTrk chunk for track %d", t);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    r.skip(4);
    const uint32_t len = r.u32();
    const size_t end = r.pos + len;
    if (!r.ok || end > r.n) {
      set_error("midi parse: track %d runs past the end of the file", t);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    // per channel: program (last change), note events in file order
    struct NoteEv {
      int64_t tick;
      int pitch, velocity;  // velocity 0 = note off
    };
    int channel_program[16] = {0};
    std::vector<int> order;  // channels in order of first note / program event
    std::vector<NoteEv> chan_ev[16];
    auto seen = [&](int c) {
      if (std::find(order.begin(), order.end(), c) == order.end()) order.push_back(c);
    };
    int64_t tick = 0;
    uint8_t running = 0;
    while (r.ok && r.pos < end) {
      tick += r.varlen();
      uint8_t st = r.u8();
      if (st < 0x80) {  // running status: this byte is the first data byte
        if (!running) {
          set_error("midi parse: running status before any status byte in track %d", t);
          return YUF_ERR_INVALID_ARGUMENT;
        }
        --r.pos;
        st = running;
      }
      const int hi = st & 0xF0, ch = st & 0x0F;
      if (hi == 0xF0) {  // meta / sysex: skipped, cancels running status
        running = 0;
        if (st == 0xFF) r.u8();
        r.skip(r.varlen());
        continue;
      }
      running = st;
      if (hi == 0x80 || hi == 0x90) {
        const int p = r.u8() & 0x7F, v = r.u8() & 0x7F;
        seen(ch);
        chan_ev[ch].push_back({tick, p, hi == 0x90 ? v : 0});
      } else if (hi == 0xC0) {
        channel_program[ch] = r.u8() & 0x7F;
        seen(ch);
      } else if (hi == 0xD0) {
        r.u8();
      } else {  // 0xA0, 0xB0, 0xE0: two data bytes
        r.u8();
        r.u8();
      }
    }
    if (!r.ok) {
      set_error("midi parse: track %d is truncated", t);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    r.pos = end;
    for (int c : order) {
      std::vector<yuf_note> done;
      std::vector<NoteEv> open;
      for (const NoteEv& e : chan_ev[c]) {
        if (e.velocity > 0) {
          open.push_back(e);
          continue;
        }
        for (size_t k = open.size(); k-- > 0;)  // the latest open note of this pitch
          if (open[k].pitch == e.pitch) {
            done.push_back({(int32_t)open[k].tick, (int32_t)std::max<int64_t>(1, e.tick - open[k].tick),
                            e.pitch, open[k].velocity});
            open.erase(open.begin() + (long)k);
            break;
          }
      }
      const int64_t last = chan_ev[c].empty() ? 0 : chan_ev[c].back().tick;
      for (const NoteEv& o : open)
        done.push_back({(int32_t)o.tick, (int32_t)std::max<int64_t>(1, last - o.tick), o.pitch, o.velocity});
      if (done.empty()) continue;
      std::stable_sort(done.begin(), done.end(), [](const yuf_note& a, const yuf_note& b) {
        if (a.start != b.start) return a.start < b.start;
        if (a.duration != b.duration) return a.duration < b.duration;
        return a.pitch < b.pitch;
      });
      tracks.push_back({channel_program[c], c == 9, std::move(done)});
    }
  }
  if (!r.ok) {
    set_error("midi parse: truncated file");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  int64_t total = 0;
  for (const Track& tr : tracks) total += (int64_t)tr.notes.size();
  *ticks_per_quarter = division;
  *n_tracks = (int)tracks.size();
  *n_notes = total;
  if (track_programs || track_is_drum) {
    if (max_tracks < (int)tracks.size() || !track_programs || !track_is_drum) {
      set_error("midi parse: %zu tracks do not fit in %d", tracks.size(), max_tracks);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    for (size_t i = 0; i < tracks.size(); ++i) {
      track_programs[i] = tracks[i].program;
      track_is_drum[i] = tracks[i].drum;
    }
  }
  if (notes) {
    if (max_notes < total || !note_track) {
      set_error("midi parse: %lld notes do not fit in %lld (or note_track is NULL)", (long long)total,
                (long long)max_notes);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    int64_t k = 0;
    for (size_t i = 0; i < tracks.size(); ++i)
      for (const yuf_note& n : tracks[i].notes) {
        notes[k] = n;
        note_track[k++] = (int32_t)i;
      }
  }
  return YUF_OK;
}

}  // extern "C"
