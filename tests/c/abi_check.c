/* A plain C99 host program against include/yufb200.h and libyufb200.so: the
 * header compiles as C, the library links, and the host-only entry points
 * (REMI codec, MIDI file I/O, status strings, host-side validation) work
 * without a GPU.  Built and run by tests/test_c_header.py. */
#include <stdio.h>
#include <string.h>

#include "yufb200.h"

#define CHECK(c)                                                          \
  do {                                                                    \
    if (!(c)) {                                                           \
      fprintf(stderr, "check failed at line %d: %s (%s)\n", __LINE__, #c, \
              yuf_last_error());                                          \
      return 1;                                                           \
    }                                                                     \
  } while (0)

int main(void) {
  /* a vocabulary with just what one note needs */
  const char* vocab[] = {"PAD_None", "Bar_None", "Position_0", "Position_4", "Program_0",
                         "Pitch_60", "Velocity_99", "Duration_0.2.8", "Duration_1.0.8"};
  yuf_remi* codec = NULL;
  CHECK(yuf_remi_create(vocab, 9, &codec) == YUF_OK);
  CHECK(yuf_remi_token_id(codec, "Pitch_60") == 5 && yuf_remi_token_id(codec, "Pitch_61") == -1);

  /* one note at tick 240 of a 480-per-quarter score, lasting a quarter */
  yuf_note note = {240, 480, 60, 100};
  yuf_track_desc track = {0, 0, "Piano", &note, 1};
  int32_t ids[16];
  int64_t n = 0;
  CHECK(yuf_remi_encode(codec, 480, &track, 1, NULL, 0, &n) == YUF_OK && n == 6);
  CHECK(yuf_remi_encode(codec, 480, &track, 1, ids, 16, &n) == YUF_OK);
  {
    const int32_t want[6] = {1, 3, 4, 5, 6, 8}; /* Bar, Position_4, Program_0, Pitch_60, Velocity_99, Duration_1.0.8 */
    CHECK(memcmp(ids, want, sizeof(want)) == 0);
  }
  int32_t prog[2], which[2];
  int nt = 0;
  int64_t nn = 0;
  yuf_note back[2];
  CHECK(yuf_remi_decode(codec, ids, n, prog, 2, &nt, back, which, 2, &nn) == YUF_OK);
  CHECK(nt == 1 && nn == 1 && prog[0] == 0 && back[0].start == 4 && back[0].duration == 8 &&
        back[0].pitch == 60 && back[0].velocity == 99);

  /* .mid bytes and back */
  uint8_t file[256];
  int64_t nb = 0;
  CHECK(yuf_midi_render(480, &track, 1, file, sizeof(file), &nb) == YUF_OK && nb > 14);
  int tpq = 0, drums[2];
  CHECK(yuf_midi_parse(file, nb, &tpq, prog, drums, 2, &nt, back, which, 2, &nn) == YUF_OK);
  CHECK(tpq == 480 && nt == 1 && nn == 1 && back[0].start == 240 && back[0].duration == 480);

  /* errors come back as status codes with a message, before any GPU work */
  CHECK(yuf_midi_parse((const uint8_t*)"not a midi file", 15, &tpq, NULL, NULL, 0, &nt, NULL, NULL, 0,
                       &nn) == YUF_ERR_INVALID_ARGUMENT);
  CHECK(strstr(yuf_last_error(), "MThd") != NULL);
  CHECK(yuf_wkv7_forward(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 1, 4, 1, 0, NULL) ==
        YUF_ERR_INVALID_ARGUMENT);
  CHECK(strcmp(yuf_status_string(YUF_ERR_UNSUPPORTED), "YUF_ERR_UNSUPPORTED") == 0);
  CHECK(yuf_abi_version() >= 1);
  yuf_remi_destroy(codec);
  printf("c abi ok\n");
  return 0;
}
