/* Stub CPU stage driver of the model-driver ABI v6.
 *
 * A stage driver the way the reference's ring loads them: a shared library built
 * with a C compiler against include/sparkpipe_b200/spark_driver_abi_v6.h (the
 * reference's v6 layout) and exporting `SparkModelDriverGetInterface`. It does no
 * math itself: the node that creates it passes a stage host (sp_stage_host, below)
 * as the node context, and each frame runs through the host, which computes the
 * stage's layers from the frame's buffers (parallel/driver_stage.py hosts the CPU
 * MLA-MoE model this way for the GPU-free plumbing run). The driver adds what the
 * ABI owns: admission, dispatch slots, completion delivery, counters.
 *
 * Programs:
 *   1 "decode"   completes later, on the driver's worker thread (external completion)
 *   2 "prefill"  completes inside submit
 * A frame runs through the node's stage host when the node context is one (see
 * sp_stage_host below): the host computes the stage from the frame's buffers. The
 * completion carries token ids from the frame's buffer in slot 7 when there is one,
 * otherwise scalar[0] + i for each new token.
 *
 * -DSP6_BREAK=N builds a variant that violates one load-time rule (for the loader's
 * fail-closed tests; never a served build):
 *   1 interface ABI version 5      2 a 63-digit SHA-256       3 two programs, one id
 *   4 validated-latency claim, no latency                     5 an unknown flag bit
 *   6 profile disagrees with the program's in-flight bound    7 no programs
 *   8 the interface symbol is missing
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include <sparkpipe_b200/spark_driver_abi_v6.h>

#ifndef SP6_BREAK
#define SP6_BREAK 0
#endif

/* The node's stage host (a convention between this test driver and its tests, not
 * part of the ABI): run() computes the stage for one frame, 0 on success. */
typedef struct sp_stage_host {
  int32_t (*run)(void* user, uint32_t program_id, const sp6_frame* frame);
  void* user;
} sp_stage_host;

#define QCAP 64

typedef struct instance {
  sp_stage_host* host;
  sp6_completion_fn complete;
  void* complete_ctx;
  sp6_wake_fn wake;
  void* wake_ctx;
  pthread_t worker;
  pthread_mutex_t mu;
  pthread_cond_t cv;
  int stop;
  sp6_completion queue[QCAP];
  unsigned head, count;
  uint64_t submitted[3], completed[3], rejected[3], admitted, generation;
} instance;

static const sp6_program_profile decode_profile = {
    sizeof(sp6_program_profile),
    (SP6_PROGRAM_STREAM_ORDERED | SP6_PROGRAM_NO_HOST_STAGING | SP6_PROGRAM_VALIDATED_LATENCY
#if SP6_BREAK == 5
     | (1u << 25)
#endif
    ),
#if SP6_BREAK == 6
    3,
#else
    4,
#endif
    64, 8, 256, 4096, 2000000,
#if SP6_BREAK == 4
    0,
#else
    1500000,
#endif
    0, 0, 0, 0, 0, 0, 0};

static const sp6_program_profile prefill_profile = {
    sizeof(sp6_program_profile), SP6_PROGRAM_BULK_PREFILL, 1, 8, 4096, 256, 4096, 0, 0, 0, 0, 0, 0, 0, 0, 0};

static sp6_status submit_decode(void* inst, sp6_frame* frame);
static sp6_status submit_prefill(void* inst, sp6_frame* frame);

static const sp6_program_descriptor programs[] = {
    {1,
     SP6_PROGRAM_EXTERNAL_COMPLETION | SP6_PROGRAM_STREAM_ORDERED | SP6_PROGRAM_NO_HOST_STAGING |
         SP6_PROGRAM_VALIDATED_LATENCY
#if SP6_BREAK == 5
         | (1u << 25)
#endif
     ,
     4, 0, "decode", &decode_profile, submit_decode},
#if SP6_BREAK == 3
    {1, SP6_PROGRAM_BULK_PREFILL, 1, 0, "prefill", &prefill_profile, submit_prefill},
#else
    {2, SP6_PROGRAM_BULK_PREFILL, 1, 0, "prefill", &prefill_profile, submit_prefill},
#endif
};

static const sp6_driver_descriptor descriptor = {
    SP6_ABI_VERSION,
    sizeof(sp6_driver_descriptor),
    "tiny-mla-moe",
    "r1",
    "stage",
    "cpu-test",
#if SP6_BREAK == 2
    "0123456789abcdef0123456789abcdef0123456789abcdef0123456789abcde",
#else
    "0123456789abcdef0123456789abcdef0123456789abcdef0123456789abcdef",
#endif
    "fedcba9876543210fedcba9876543210fedcba9876543210fedcba9876543210",
#if SP6_BREAK == 7
    0,
#else
    2,
#endif
    1,
    programs};

/* Completion of one frame: tokens from buffer slot 7 if present, else scalar[0] + i. */
static void fill_completion(const sp6_frame* f, sp6_completion* c, sp6_status status) {
  memset(c, 0, sizeof(*c));
  c->request_id = f->request_id;
  c->sequence_id = f->sequence_id;
  c->sequence_position = f->sequence_position;
  c->program_id = f->program_id;
  c->driver_dispatch_slot = f->driver_dispatch_slot;
  c->status = status;
  c->completion_flags = SP6_COMPLETION_FLAG_TOKEN_IDS;
  const uint32_t* tokens = 0;
  uint32_t n = f->new_token_count < SP6_COMPLETION_TOKENS ? f->new_token_count : SP6_COMPLETION_TOKENS;
  for (uint32_t i = 0; i < f->buffer_count; ++i)
    if (f->buffers[i].slot == 7 && f->buffers[i].address) {
      tokens = (const uint32_t*)f->buffers[i].address;
      if (f->buffers[i].bytes / 4 < n) n = (uint32_t)(f->buffers[i].bytes / 4);
    }
  for (uint32_t i = 0; i < n; ++i) c->token_ids[i] = tokens ? tokens[i] : (uint32_t)(f->scalar[0] + i);
  c->token_count = n;
  c->accepted_token_count = n;
  c->residency = f->residency;
}

static sp6_status run_stage(instance* in, const sp6_frame* f) {
  if (!in->host || !in->host->run) return 0;
  return in->host->run(in->host->user, f->program_id, f) == 0 ? 0 : 17 /* internal error */;
}

static void* worker(void* arg) {
  instance* in = (instance*)arg;
  pthread_mutex_lock(&in->mu);
  for (;;) {
    while (!in->stop && in->count == 0) pthread_cond_wait(&in->cv, &in->mu);
    if (in->count == 0 && in->stop) break;
    sp6_completion c = in->queue[in->head];
    in->head = (in->head + 1) % QCAP;
    in->count--;
    in->completed[1]++;
    pthread_mutex_unlock(&in->mu);
    in->complete(in->complete_ctx, &c);
    if (in->wake) in->wake(in->wake_ctx);
    pthread_mutex_lock(&in->mu);
  }
  pthread_mutex_unlock(&in->mu);
  return 0;
}

static sp6_status submit_decode(void* inst, sp6_frame* f) {
  instance* in = (instance*)inst;
  /* the stage runs now (on the caller's thread); its completion is reported later */
  const sp6_status st = run_stage(in, f);
  sp6_completion c;
  fill_completion(f, &c, st);
  pthread_mutex_lock(&in->mu);
  if (in->count == QCAP) {
    in->rejected[1]++;
    pthread_mutex_unlock(&in->mu);
    return 15; /* busy */
  }
  in->queue[(in->head + in->count) % QCAP] = c;
  in->count++;
  in->submitted[1]++;
  pthread_cond_signal(&in->cv);
  pthread_mutex_unlock(&in->mu);
  return 0;
}

static sp6_status submit_prefill(void* inst, sp6_frame* f) {
  instance* in = (instance*)inst;
  const sp6_status st = run_stage(in, f);
  sp6_completion c;
  fill_completion(f, &c, st);
  pthread_mutex_lock(&in->mu);
  in->submitted[2]++;
  in->completed[2]++;
  pthread_mutex_unlock(&in->mu);
  f->completion_function(f->completion_context, &c);
  return 0;
}

static sp6_status create(const sp6_create_request* req, void** out) {
  if (!req || !out || !req->completion_function) return 1; /* invalid argument */
  instance* in = (instance*)calloc(1, sizeof(instance));
  if (!in) return 2;
  in->host = (sp_stage_host*)req->node_context;
  in->complete = req->completion_function;
  in->complete_ctx = req->completion_context;
  in->wake = req->wake_function;
  in->wake_ctx = req->wake_context;
  pthread_mutex_init(&in->mu, 0);
  pthread_cond_init(&in->cv, 0);
  if (pthread_create(&in->worker, 0, worker, in) != 0) {
    free(in);
    return 2;
  }
  *out = in;
  return 0;
}

static void destroy(void* inst) {
  instance* in = (instance*)inst;
  if (!in) return;
  pthread_mutex_lock(&in->mu);
  in->stop = 1;
  pthread_cond_signal(&in->cv);
  pthread_mutex_unlock(&in->mu);
  pthread_join(in->worker, 0); /* queued completions are delivered first */
  pthread_cond_destroy(&in->cv);
  pthread_mutex_destroy(&in->mu);
  free(in);
}

static sp6_status admit(void* inst, const sp6_admission_request* r, sp6_admission_decision* d) {
  instance* in = (instance*)inst;
  if (!r || !d || r->program_id < 1 || r->program_id > 2) return 1;
  const sp6_program_profile* p = r->program_id == 1 ? &decode_profile : &prefill_profile;
  pthread_mutex_lock(&in->mu);
  d->accepted = 1;
  d->rejection_reason = SP6_ADMIT_ACCEPTED;
  if (r->active_slot_count > p->max_active_slots) {
    d->accepted = 0;
    d->rejection_reason = SP6_ADMIT_KV_CAPACITY;
  } else if (r->new_token_count > p->max_new_tokens) {
    d->accepted = 0;
    d->rejection_reason = SP6_ADMIT_UNSUPPORTED_SHAPE;
  } else if (r->program_id == 1 && in->count >= decode_profile.max_inflight) {
    d->accepted = 0;
    d->rejection_reason = SP6_ADMIT_BUSY;
  }
  if (d->accepted) {
    in->admitted++;
    d->driver_dispatch_slot = (uint32_t)(in->admitted % 4);
    d->driver_dispatch_generation = ++in->generation;
    d->driver_dispatch_cookie0 = r->request_id ^ 0x5a5a5a5aull;
    d->driver_dispatch_cookie1 = r->sequence_id;
  } else {
    d->driver_dispatch_slot = SP6_INVALID_DISPATCH_SLOT;
  }
  d->estimated_service_time_ns = r->program_id == 1 ? decode_profile.validated_latency_ns : 0;
  d->available_dispatch_slot_count = QCAP - in->count;
  pthread_mutex_unlock(&in->mu);
  return 0;
}

static sp6_status snapshot(void* inst, uint32_t program_id, sp6_runtime_snapshot* s) {
  instance* in = (instance*)inst;
  if (!s || program_id < 1 || program_id > 2) return 1;
  pthread_mutex_lock(&in->mu);
  s->program_id = program_id;
  s->submitted_count = in->submitted[program_id];
  s->completed_count = in->completed[program_id];
  s->rejected_count = in->rejected[program_id];
  s->active_submission_count = program_id == 1 ? in->count : 0;
  s->available_dispatch_slot_count = QCAP - in->count;
  s->host_callback_completion_count = in->completed[1] + in->completed[2];
  pthread_mutex_unlock(&in->mu);
  return 0;
}

static const sp6_interface iface = {
#if SP6_BREAK == 1
    5,
#else
    SP6_ABI_VERSION,
#endif
    sizeof(sp6_interface), &descriptor, create, destroy, admit, snapshot};

#if SP6_BREAK == 8
__attribute__((visibility("default"))) const sp6_interface* SparkModelDriverGetInterfaceX(void) { return &iface; }
#else
__attribute__((visibility("default"))) const sp6_interface* SparkModelDriverGetInterface(void) { return &iface; }
#endif
