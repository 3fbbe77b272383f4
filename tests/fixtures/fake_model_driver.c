/* Minimal valid model driver for the loader tests: one host program that echoes its
 * input reversed and counts submissions. Built by the tests with the system C
 * compiler; -DSPB_FAKE_BREAK=<n> produces deliberately invalid variants. */
#include <sparkpipe_b200/model_driver.h>
#include <stdlib.h>
#include <string.h>

#ifndef SPB_FAKE_BREAK
#define SPB_FAKE_BREAK 0
#endif
#ifndef SPB_FAKE_TARGET
#define SPB_FAKE_TARGET "host.cpu"
#endif

typedef struct fake_instance {
  uint64_t submits;
} fake_instance;

static int32_t fake_submit(void* inst, const spb_buffer* in, spb_buffer* out) {
  fake_instance* f = (fake_instance*)inst;
  if (out->bytes < in->bytes) return 2; /* capacity exceeded */
  const char* s = (const char*)in->data;
  char* d = (char*)out->data;
  for (uint64_t i = 0; i < in->bytes; ++i) d[i] = s[in->bytes - 1 - i];
  out->bytes = in->bytes;
  f->submits++;
  return 0;
}

static const spb_program_profile fake_profiles[2] = {
    {sizeof(spb_program_profile),
     SPB_PROGRAM_STREAM_ORDERED | SPB_PROGRAM_NO_DEVICE_MEMCPY | (SPB_FAKE_BREAK == 3 ? SPB_PROGRAM_VALIDATED_LATENCY : 0),
     1, 0, 4096, 0, SPB_FAKE_BREAK == 3 ? 0 : 1000, 0},
    {sizeof(spb_program_profile), SPB_PROGRAM_STREAM_ORDERED, 2, 0, 0, 0, 0, 0},
};

static const spb_program_descriptor fake_programs[2] = {
    {1, SPB_PROGRAM_STREAM_ORDERED | SPB_PROGRAM_NO_DEVICE_MEMCPY | (SPB_FAKE_BREAK == 3 ? SPB_PROGRAM_VALIDATED_LATENCY : 0),
     1, 0, "fixture_program", &fake_profiles[0], fake_submit},
    {SPB_FAKE_BREAK == 4 ? 1 : 2, SPB_PROGRAM_STREAM_ORDERED, 2, 0, "fixture_program_b", &fake_profiles[1], fake_submit},
};

static const spb_model_driver_descriptor fake_descriptor = {
    SPB_MODEL_DRIVER_ABI_VERSION,
    sizeof(spb_model_driver_descriptor),
    "fixture-model",
    "r1",
    "stage0",
    SPB_FAKE_TARGET,
    "0123456789abcdef0123456789abcdef0123456789abcdef0123456789abcdef",
    SPB_FAKE_BREAK == 2 ? "not-a-hash" : "fedcba9876543210fedcba9876543210fedcba9876543210fedcba9876543210",
    2,
    1,
    fake_programs,
};

static int32_t fake_create(const char* config, void** inst) {
  (void)config;
  fake_instance* f = (fake_instance*)calloc(1, sizeof(fake_instance));
  if (!f) return 17;
  *inst = f;
  return 0;
}
static void fake_destroy(void* inst) { free(inst); }
static int32_t fake_admit(void* inst, spb_admission* a) {
  (void)inst;
  a->accepted = a->sequences > 4 ? 4 : a->sequences;
  return 0;
}
static int32_t fake_snapshot(void* inst, spb_snapshot* s) {
  s->submits = ((fake_instance*)inst)->submits;
  s->completions = s->submits;
  s->inflight = 0;
  s->reserved = 0;
  return 0;
}

static const spb_model_driver_interface fake_interface = {
    SPB_FAKE_BREAK == 1 ? 99u : SPB_MODEL_DRIVER_ABI_VERSION,
    sizeof(spb_model_driver_interface),
    &fake_descriptor,
    fake_create,
    fake_destroy,
    fake_admit,
    fake_snapshot,
};

#if SPB_FAKE_BREAK != 5
const spb_model_driver_interface* spb_model_driver_get_interface(void) { return &fake_interface; }
#else
const spb_model_driver_interface* some_other_symbol(void) { return &fake_interface; }
#endif
