/* Binary-compatible view of the reference's model-driver ABI, version 6.
 *
 * A stage driver built for the reference (a shared library exporting
 * `SparkModelDriverGetInterface`, ABI version 6) loads in this framework through
 * `csrc/core/driver_v6.cpp`. The loader never sees the reference's header: this
 * header declares the same structs field for field, so the in-memory layout (LP64)
 * and the exported symbol name are identical, which is what a compiled driver and
 * its loader have to agree on. The type and macro names here are this framework's
 * own (`sp6_*`, `SP6_*`); the numeric constants (ABI version, flag bits, admission
 * reasons, capacities) are the ABI's and must not change.
 *
 * Reference: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_model_driver.h:12-255
 * (declarations), crates/spark-sys/src/driver.rs (load-time validation rules).
 *
 * The status type is a 32-bit enum with the reference's numbering (0 = ok; see
 * csrc/core/common.h `Status`).
 */
#ifndef SPARKPIPE_B200_SPARK_DRIVER_ABI_V6_H
#define SPARKPIPE_B200_SPARK_DRIVER_ABI_V6_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SP6_ABI_VERSION 6u
#define SP6_INTERFACE_SYMBOL "SparkModelDriverGetInterface"
#define SP6_COMPLETION_TOKENS 8u
#define SP6_COMPLETION_DRAFT_TOKENS 8u
#define SP6_COMPLETION_FLAG_TOKEN_IDS 0x00000001u
#define SP6_COMPLETION_FLAG_DRAFT_TOKEN_IDS 0x00000002u

/* program flags (bit values fixed by the ABI) */
#define SP6_PROGRAM_EXTERNAL_COMPLETION 0x00000001u
#define SP6_PROGRAM_STREAM_ORDERED 0x00000002u
#define SP6_PROGRAM_DRIVER_OWNS_RESIDENT_STATE 0x00000004u
#define SP6_PROGRAM_DRIVER_OWNS_KV_CACHE 0x00000008u
#define SP6_PROGRAM_JIT_KV_CACHE 0x00000010u
#define SP6_PROGRAM_ZERO_COPY_NODE_CONTEXT 0x00000020u
#define SP6_PROGRAM_PRIVATE_QUEUE_PRESSURE 0x00000040u
#define SP6_PROGRAM_NO_HOST_STAGING 0x00000080u
#define SP6_PROGRAM_FIXED_FIRMWARE 0x00000100u
#define SP6_PROGRAM_VALIDATED_LATENCY 0x00000200u
#define SP6_PROGRAM_CAPTURED_CUDA_GRAPH 0x00000400u
#define SP6_PROGRAM_NO_DEVICE_MEMCPY 0x00000800u
#define SP6_PROGRAM_DRIVER_PRIVATE_EXPERT_QUEUES 0x00001000u
#define SP6_PROGRAM_STREAM_EVENT_DEPENDENCIES 0x00002000u
#define SP6_PROGRAM_RESIDENCY_AFFINITY_REQUIRED 0x00004000u
#define SP6_PROGRAM_BATCH_SHAPE_FIXED 0x00008000u
#define SP6_PROGRAM_REQUIRES_HIDDEN_TRANSPORT 0x00010000u
#define SP6_PROGRAM_NO_FILE_TRANSPORT 0x00020000u
#define SP6_PROGRAM_NO_SHELL_TRANSPORT 0x00040000u
#define SP6_PROGRAM_BULK_PREFILL 0x00080000u
#define SP6_PROGRAM_KNOWN_FLAGS 0x000fffffu /* the twenty bits above */

#define SP6_BUFFER_READ 0x00000001u
#define SP6_BUFFER_WRITE 0x00000002u
#define SP6_FRAME_DISPATCH_SLOT_VALID 0x00000001u
#define SP6_FRAME_PREFILL 0x00000002u
#define SP6_SCALARS 8u
#define SP6_INVALID_DISPATCH_SLOT 0xffffffffu

/* admission rejection reasons */
#define SP6_ADMIT_ACCEPTED 0u
#define SP6_ADMIT_BUSY 1u
#define SP6_ADMIT_KV_CAPACITY 2u
#define SP6_ADMIT_DEADLINE 3u
#define SP6_ADMIT_HOST_STAGING_REQUIRED 4u
#define SP6_ADMIT_UNSUPPORTED_SHAPE 5u

typedef int32_t sp6_status; /* an enum in C: four bytes, 0 = ok */

typedef struct sp6_buffer {
  uint32_t slot;
  uint32_t flags;
  void* address;
  uint64_t bytes;
} sp6_buffer;

typedef struct sp6_residency {
  uint64_t word0, word1, generation, owner;
} sp6_residency;

typedef struct sp6_completion {
  uint64_t request_id;
  uint64_t sequence_id;
  uint64_t sequence_position;
  uint32_t program_id;
  uint32_t driver_dispatch_slot;
  uint32_t accepted_token_count;
  uint32_t completion_flags;
  uint32_t token_count;
  uint32_t token_ids[SP6_COMPLETION_TOKENS];
  uint32_t draft_token_count;
  uint32_t draft_token_ids[SP6_COMPLETION_DRAFT_TOKENS];
  sp6_status status;
  sp6_residency residency;
  uint64_t queue_delay_ns;
  uint64_t service_time_ns;
  uint64_t device_memcpy_bytes;
  uint64_t host_staging_bytes;
} sp6_completion;

typedef void (*sp6_completion_fn)(void* completion_context, const sp6_completion* completion);
typedef void (*sp6_wake_fn)(void* wake_context);

typedef struct sp6_frame {
  uint64_t request_id;
  uint64_t sequence_id;
  uint64_t sequence_position;
  uint64_t deadline_time_ns;
  uint32_t active_slot_count;
  uint32_t new_token_count;
  uint32_t priority;
  uint32_t flags;
  uint32_t driver_dispatch_slot;
  uint32_t program_id;
  uint64_t driver_dispatch_generation;
  uint64_t driver_dispatch_cookie0;
  uint64_t driver_dispatch_cookie1;
  void* execution_stream;
  sp6_buffer* buffers;
  uint32_t buffer_count;
  uint32_t reserved;
  uint64_t scalar[SP6_SCALARS];
  sp6_residency residency;
  void* user_context;
  sp6_completion_fn completion_function;
  void* completion_context;
} sp6_frame;

typedef struct sp6_program_profile {
  uint32_t descriptor_bytes;
  uint32_t profile_flags;
  uint32_t max_inflight;
  uint32_t max_active_slots;
  uint32_t max_new_tokens;
  uint32_t max_resident_sequences;
  uint64_t max_sequence_tokens;
  uint64_t target_latency_ns;
  uint64_t validated_latency_ns;
  uint64_t resident_weight_bytes;
  uint64_t resident_kv_bytes;
  uint64_t static_workspace_bytes;
  uint64_t device_memcpy_bytes_per_submit_ceiling;
  uint64_t host_staging_bytes_per_submit_ceiling;
  uint32_t private_queue_count;
  uint32_t reserved;
} sp6_program_profile;

typedef struct sp6_admission_request {
  uint32_t descriptor_bytes;
  uint32_t program_id;
  uint64_t request_id;
  uint64_t sequence_id;
  uint64_t sequence_position;
  uint64_t deadline_time_ns;
  uint32_t active_slot_count;
  uint32_t new_token_count;
  uint32_t priority;
  uint32_t frame_flags;
  sp6_residency residency;
} sp6_admission_request;

typedef struct sp6_admission_decision {
  uint32_t descriptor_bytes;
  uint32_t accepted;
  uint32_t rejection_reason;
  uint32_t driver_dispatch_slot;
  uint64_t estimated_queue_delay_ns;
  uint64_t estimated_service_time_ns;
  uint64_t endpoint_cost;
  uint64_t residency_match_score;
  uint64_t device_memcpy_bytes;
  uint64_t host_staging_bytes;
  uint32_t private_queue_pressure;
  uint32_t available_dispatch_slot_count;
  uint64_t driver_dispatch_generation;
  uint64_t driver_dispatch_cookie0;
  uint64_t driver_dispatch_cookie1;
} sp6_admission_decision;

typedef struct sp6_runtime_snapshot {
  uint32_t descriptor_bytes;
  uint32_t program_id;
  uint32_t active_submission_count;
  uint32_t available_dispatch_slot_count;
  uint64_t submitted_count;
  uint64_t completed_count;
  uint64_t rejected_count;
  uint64_t resident_sequence_count;
  uint64_t resident_token_count;
  uint64_t kv_token_capacity;
  uint64_t device_memcpy_bytes_per_submit;
  uint64_t host_staging_bytes_per_submit;
  uint64_t cuda_graph_capture_count;
  uint64_t cuda_graph_replay_count;
  uint64_t host_callback_completion_count;
  uint64_t stale_admission_count;
  uint32_t private_queue_pressure;
  uint32_t reserved;
} sp6_runtime_snapshot;

typedef struct sp6_create_request {
  const char* node_id;
  const char* node_target;
  void* node_context;
  sp6_completion_fn completion_function;
  void* completion_context;
  sp6_wake_fn wake_function;
  void* wake_context;
} sp6_create_request;

typedef sp6_status (*sp6_submit_fn)(void* driver_instance, sp6_frame* frame);

typedef struct sp6_program_descriptor {
  uint32_t program_id;
  uint32_t flags;
  uint32_t max_inflight;
  uint32_t reserved;
  const char* name;
  const sp6_program_profile* profile;
  sp6_submit_fn submit;
} sp6_program_descriptor;

typedef struct sp6_driver_descriptor {
  uint32_t abi_version;
  uint32_t descriptor_bytes;
  const char* model_id;
  const char* model_revision;
  const char* stage_name;
  const char* target;
  const char* model_description_sha256;
  const char* compiled_program_sha256;
  uint32_t program_count;
  uint32_t module_instance_count;
  const sp6_program_descriptor* programs;
} sp6_driver_descriptor;

typedef struct sp6_interface {
  uint32_t abi_version;
  uint32_t interface_bytes;
  const sp6_driver_descriptor* descriptor;
  sp6_status (*create)(const sp6_create_request* request, void** driver_instance);
  void (*destroy)(void* driver_instance);
  sp6_status (*admit)(void* driver_instance, const sp6_admission_request* request, sp6_admission_decision* decision);
  sp6_status (*snapshot)(void* driver_instance, uint32_t program_id, sp6_runtime_snapshot* snapshot);
} sp6_interface;

typedef const sp6_interface* (*sp6_get_interface_fn)(void);

/* LP64 layout of the ABI (the sizes every v6 driver is compiled with). */
#if defined(__LP64__) || defined(_LP64)
#ifdef __cplusplus
#define SP6_STATIC_ASSERT static_assert
#else
#define SP6_STATIC_ASSERT _Static_assert
#endif
SP6_STATIC_ASSERT(sizeof(sp6_buffer) == 24, "sp6_buffer");
SP6_STATIC_ASSERT(sizeof(sp6_residency) == 32, "sp6_residency");
SP6_STATIC_ASSERT(sizeof(sp6_completion) == 184, "sp6_completion");
SP6_STATIC_ASSERT(offsetof(sp6_completion, status) == 112, "sp6_completion.status");
SP6_STATIC_ASSERT(sizeof(sp6_frame) == 224, "sp6_frame");
SP6_STATIC_ASSERT(offsetof(sp6_frame, scalar) == 104, "sp6_frame.scalar");
SP6_STATIC_ASSERT(sizeof(sp6_program_profile) == 96, "sp6_program_profile");
SP6_STATIC_ASSERT(sizeof(sp6_admission_request) == 88, "sp6_admission_request");
SP6_STATIC_ASSERT(sizeof(sp6_admission_decision) == 96, "sp6_admission_decision");
SP6_STATIC_ASSERT(sizeof(sp6_runtime_snapshot) == 120, "sp6_runtime_snapshot");
SP6_STATIC_ASSERT(sizeof(sp6_create_request) == 56, "sp6_create_request");
SP6_STATIC_ASSERT(sizeof(sp6_program_descriptor) == 40, "sp6_program_descriptor");
SP6_STATIC_ASSERT(sizeof(sp6_driver_descriptor) == 72, "sp6_driver_descriptor");
SP6_STATIC_ASSERT(sizeof(sp6_interface) == 48, "sp6_interface");
#undef SP6_STATIC_ASSERT
#endif

#ifdef __cplusplus
}
#endif

#endif /* SPARKPIPE_B200_SPARK_DRIVER_ABI_V6_H */
