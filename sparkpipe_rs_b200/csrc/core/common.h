// Shared definitions of the C++ serving runtime: the status space and the
// FNV-1a hashing used for content addressing and packet fingerprints.
//
// The status codes keep the numeric values of the reference's SparkStatus
// (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_status.h:10-29) so
// statuses carried in wire records stay interoperable.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

namespace spc {

enum class Status : uint32_t {
  Ok = 0,
  InvalidArgument,
  CapacityExceeded,
  NotFound,
  IoError,
  ParseError,
  SchemaError,
  HashMismatch,
  ModuleNotValidated,
  ValidationFailed,
  AbiMismatch,
  TargetMismatch,
  CompilerError,
  DriverLoadError,
  RouteNotFound,
  Busy,
  Duplicate,
  InternalError,
  Pending,
  Unsupported,
};

inline const char* status_name(Status s) {
  switch (s) {
    case Status::Ok: return "ok";
    case Status::InvalidArgument: return "invalid_argument";
    case Status::CapacityExceeded: return "capacity_exceeded";
    case Status::NotFound: return "not_found";
    case Status::IoError: return "io_error";
    case Status::ParseError: return "parse_error";
    case Status::SchemaError: return "schema_error";
    case Status::HashMismatch: return "hash_mismatch";
    case Status::ModuleNotValidated: return "module_not_validated";
    case Status::ValidationFailed: return "validation_failed";
    case Status::AbiMismatch: return "abi_mismatch";
    case Status::TargetMismatch: return "target_mismatch";
    case Status::CompilerError: return "compiler_error";
    case Status::DriverLoadError: return "driver_load_error";
    case Status::RouteNotFound: return "route_not_found";
    case Status::Busy: return "busy";
    case Status::Duplicate: return "duplicate";
    case Status::InternalError: return "internal_error";
    case Status::Pending: return "pending";
    case Status::Unsupported: return "unsupported";
  }
  return "unknown";
}

// Exception carrying a Status; the Python bindings translate it to
// sparkpipe_rs_b200.core.StatusError with the same code.
struct StatusError : std::runtime_error {
  Status status;
  StatusError(Status s, const std::string& what) : std::runtime_error(what), status(s) {}
};

[[noreturn]] inline void fail(Status s, const std::string& what) { throw StatusError(s, what); }

// ------------------------------------------------------------------ FNV-1a
constexpr uint64_t kFnv64Offset = 1469598103934665603ull;
constexpr uint64_t kFnv64Prime = 1099511628211ull;
constexpr uint32_t kFnv32Offset = 2166136261u;
constexpr uint32_t kFnv32Prime = 16777619u;

inline uint64_t fnv1a64(const void* data, size_t n, uint64_t h = kFnv64Offset) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= kFnv64Prime;
  }
  return h;
}

inline uint32_t fnv1a32(const void* data, size_t n, uint32_t h = kFnv32Offset) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= kFnv32Prime;
  }
  return h;
}

// Little-endian field writers/readers for the fixed-layout wire records.
inline void put_u32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = uint8_t(v >> (8 * i));
}
inline void put_u64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = uint8_t(v >> (8 * i));
}
inline uint32_t get_u32(const uint8_t* p) {
  uint32_t v = 0;
  for (int i = 0; i < 4; ++i) v |= uint32_t(p[i]) << (8 * i);
  return v;
}
inline uint64_t get_u64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= uint64_t(p[i]) << (8 * i);
  return v;
}

}  // namespace spc
