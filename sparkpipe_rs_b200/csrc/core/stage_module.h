// Common services of a stage module (a model driver instance that owns device
// memory and dispatch slots):
//
//   DeviceLedger   every device allocation of a module with its size (at most
//                  4096), rolled back to a mark when a load fails half way and
//                  released in reverse order on destroy, so a failed or destroyed
//                  module leaks nothing. Allocation goes through an Allocator (the
//                  CUDA one from Python, or host memory in tests).
//   pack regions   a weight pack file read at an offset into host memory, or into a
//                  fresh ledger allocation through 64 MB pinned-size staging chunks.
//   SlotTable      dispatch slots as atomic states: lock-free claim / release, an
//                  all-or-nothing claim of an index set, counts, and the quiesce
//                  wait of destroy (every slot free, bounded: 30 s by default).
//   environment    typed, range-checked environment settings.
//   admission      the driver ABI's admission record filled from slot availability.
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_stage_module_common.h:8-117
// (allocation cap, staging chunk size, slot states, destroy quiesce timeout, the set
// of services). The implementation is this framework's own.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace stm {

constexpr uint32_t kMaxDeviceAllocations = 4096;
constexpr uint64_t kStagingChunkBytes = 64ull << 20;
constexpr uint32_t kSlotFree = 0;
constexpr uint32_t kSlotClaimed = 1;
constexpr uint64_t kQuiesceTimeoutNs = 30000000000ull;

class Allocator {
 public:
  virtual ~Allocator() = default;
  virtual Status allocate(uint64_t bytes, void** ptr) = 0;
  virtual void release(void* ptr) = 0;
  virtual Status zero(void* ptr, uint64_t bytes) = 0;
  virtual Status copy_from_host(void* dst, const void* src, uint64_t bytes) = 0;
};

// Host memory standing in for a device (tests, CPU stages).
class HostAllocator : public Allocator {
 public:
  Status allocate(uint64_t bytes, void** ptr) override;
  void release(void* ptr) override;
  Status zero(void* ptr, uint64_t bytes) override;
  Status copy_from_host(void* dst, const void* src, uint64_t bytes) override;
};

class DeviceLedger {
 public:
  DeviceLedger(std::string module_tag, std::shared_ptr<Allocator> alloc);
  ~DeviceLedger();
  DeviceLedger(const DeviceLedger&) = delete;
  DeviceLedger& operator=(const DeviceLedger&) = delete;

  void* allocate(uint64_t bytes, bool zeroed = false);
  // Releases (newest first) every allocation made after the first `count`.
  void rollback(uint32_t count);
  void release_all() { rollback(0); }
  uint32_t count() const { return (uint32_t)ptrs_.size(); }
  uint64_t bytes_resident() const { return resident_; }
  const std::string& tag() const { return tag_; }
  Allocator& allocator() { return *alloc_; }

 private:
  std::string tag_;
  std::shared_ptr<Allocator> alloc_;
  std::vector<void*> ptrs_;
  std::vector<uint64_t> sizes_;
  uint64_t resident_ = 0;
};

// Reads `bytes` at `offset` of a pack file into host memory.
void pack_read(const std::string& tag, std::FILE* f, uint64_t offset, void* dst, uint64_t bytes);
// Reads a pack region into a new ledger allocation through staging chunks;
// returns the device pointer. A failure rolls the allocation back.
void* load_device_region(DeviceLedger& ledger, std::FILE* f, uint64_t offset, uint64_t bytes);

class SlotTable {
 public:
  explicit SlotTable(uint32_t slots);
  // Claims the lowest free slot; false when every slot is claimed.
  bool claim(uint32_t* index);
  void release(uint32_t index);
  // Claims every index of the set, or none (Busy when one is taken).
  Status claim_set(const std::vector<uint32_t>& indices);
  void release_set(const std::vector<uint32_t>& indices);
  uint32_t free_count() const;
  uint32_t size() const { return (uint32_t)states_.size(); }
  bool claimed(uint32_t index) const;
  // Waits until every slot is free (the destroy quiesce); Ok, or Busy on timeout.
  Status wait_all_free(uint64_t timeout_ns = kQuiesceTimeoutNs) const;

 private:
  std::vector<std::atomic<uint32_t>> states_;
};

std::string env_text(const std::string& tag, const std::string& name, const std::string& fallback);
uint64_t env_unsigned(const std::string& tag, const std::string& name, uint64_t minimum, uint64_t maximum,
                      uint64_t fallback);

}  // namespace stm
}  // namespace spc
