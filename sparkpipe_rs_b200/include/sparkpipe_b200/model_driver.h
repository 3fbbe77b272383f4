/* Model-driver ABI of sparkpipe_rs_b200 (C, stable across compilers).
 *
 * A model driver is a shared library exporting one symbol,
 * `spb_model_driver_get_interface`, that returns a pointer to a static
 * `spb_model_driver_interface`. The interface names the driver's descriptor (model
 * identity, revision, stage, compile target, content hashes, program table) and its
 * entry points (create / destroy / admit / snapshot; one submit per program). The
 * loader (`csrc/core/driver_loader.cpp`) validates everything fail-closed before any
 * entry point is called: ABI version and struct sizes, non-empty identity strings,
 * 64-hex-digit SHA-256 fields, non-empty unique program table, known program flags,
 * per-program profiles agreeing with their programs, flag claims backed by profile
 * numbers, and the compile target against the node's.
 *
 * Concepts follow the reference's driver ABI
 * (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_model_driver.h:12-255,
 * loader crates/spark-sys/src/driver.rs); this header, its names and its layout are
 * this framework's own. All structs are laid out for LP64 (checked below).
 */
#ifndef SPARKPIPE_B200_MODEL_DRIVER_H
#define SPARKPIPE_B200_MODEL_DRIVER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPB_MODEL_DRIVER_ABI_VERSION 1u
#define SPB_MODEL_DRIVER_SYMBOL "spb_model_driver_get_interface"

/* program flags */
#define SPB_PROGRAM_EXTERNAL_COMPLETION 0x00000001u   /* completes through a callback, not on return */
#define SPB_PROGRAM_STREAM_ORDERED 0x00000002u        /* work is ordered on the caller's CUDA stream */
#define SPB_PROGRAM_OWNS_RESIDENT_STATE 0x00000004u
#define SPB_PROGRAM_OWNS_KV_CACHE 0x00000008u
#define SPB_PROGRAM_CAPTURED_CUDA_GRAPH 0x00000010u    /* replays a captured CUDA graph */
#define SPB_PROGRAM_NO_HOST_STAGING 0x00000020u        /* claim: no host staging bytes per submit */
#define SPB_PROGRAM_NO_DEVICE_MEMCPY 0x00000040u       /* claim: no device memcpy bytes per submit */
#define SPB_PROGRAM_VALIDATED_LATENCY 0x00000080u      /* claim: a measured latency is recorded */
#define SPB_PROGRAM_PRIVATE_QUEUES 0x00000100u         /* claim: private work queues exist */
#define SPB_PROGRAM_BATCH_SHAPE_FIXED 0x00000200u
#define SPB_PROGRAM_BULK_PREFILL 0x00000400u
#define SPB_PROGRAM_PEER_MEMORY 0x00000800u            /* uses NVLink peer memory of other ranks */
#define SPB_PROGRAM_KNOWN_FLAGS 0x00000fffu

typedef struct spb_buffer {
  void* data;
  uint64_t bytes;
} spb_buffer;

typedef struct spb_program_profile {
  uint32_t descriptor_bytes; /* sizeof(spb_program_profile) */
  uint32_t profile_flags;    /* program flags minus SPB_PROGRAM_EXTERNAL_COMPLETION */
  uint32_t max_inflight;     /* equals the program's */
  uint32_t private_queue_count;
  uint64_t host_staging_bytes_ceiling;
  uint64_t device_memcpy_bytes_ceiling;
  uint64_t validated_latency_ns;
  uint64_t reserved; /* zero */
} spb_program_profile;

typedef int32_t (*spb_submit_fn)(void* instance, const spb_buffer* input, spb_buffer* output);

typedef struct spb_program_descriptor {
  uint32_t program_id; /* nonzero, unique */
  uint32_t flags;
  uint32_t max_inflight; /* nonzero */
  uint32_t reserved;     /* zero */
  const char* name;      /* non-empty, unique */
  const spb_program_profile* profile;
  spb_submit_fn submit;
} spb_program_descriptor;

typedef struct spb_model_driver_descriptor {
  uint32_t abi_version;
  uint32_t descriptor_bytes;
  const char* model_id;
  const char* model_revision;
  const char* stage_name;
  const char* target; /* e.g. "sm_100a.b200", "host.cpu" */
  const char* model_description_sha256; /* 64 hex digits */
  const char* compiled_program_sha256;  /* 64 hex digits */
  uint32_t program_count;
  uint32_t module_instance_count;
  const spb_program_descriptor* programs;
} spb_model_driver_descriptor;

typedef struct spb_admission {
  uint32_t program_id;
  uint32_t sequences;
  uint32_t tokens;
  uint32_t accepted; /* out */
} spb_admission;

typedef struct spb_snapshot {
  uint64_t submits;
  uint64_t completions;
  uint64_t inflight;
  uint64_t reserved;
} spb_snapshot;

typedef struct spb_model_driver_interface {
  uint32_t abi_version;
  uint32_t interface_bytes;
  const spb_model_driver_descriptor* descriptor;
  int32_t (*create)(const char* config_json, void** instance);
  void (*destroy)(void* instance);
  int32_t (*admit)(void* instance, spb_admission* request);
  int32_t (*snapshot)(void* instance, spb_snapshot* out);
} spb_model_driver_interface;

typedef const spb_model_driver_interface* (*spb_get_interface_fn)(void);

#if defined(__cplusplus)
#define SPB_STATIC_ASSERT(c, m) static_assert(c, m)
#else
#define SPB_STATIC_ASSERT(c, m) _Static_assert(c, m)
#endif
SPB_STATIC_ASSERT(sizeof(void*) == 8, "LP64 only");
SPB_STATIC_ASSERT(sizeof(spb_buffer) == 16, "spb_buffer layout");
SPB_STATIC_ASSERT(sizeof(spb_program_profile) == 48, "spb_program_profile layout");
SPB_STATIC_ASSERT(sizeof(spb_program_descriptor) == 40, "spb_program_descriptor layout");
SPB_STATIC_ASSERT(offsetof(spb_program_descriptor, name) == 16, "spb_program_descriptor.name offset");
SPB_STATIC_ASSERT(sizeof(spb_model_driver_descriptor) == 72, "spb_model_driver_descriptor layout");
SPB_STATIC_ASSERT(offsetof(spb_model_driver_descriptor, programs) == 64, "descriptor.programs offset");
SPB_STATIC_ASSERT(sizeof(spb_admission) == 16, "spb_admission layout");
SPB_STATIC_ASSERT(sizeof(spb_snapshot) == 32, "spb_snapshot layout");
SPB_STATIC_ASSERT(sizeof(spb_model_driver_interface) == 48, "spb_model_driver_interface layout");

#ifdef __cplusplus
}
#endif
#endif /* SPARKPIPE_B200_MODEL_DRIVER_H */
