#include "stage_module.h"

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

namespace spc {
namespace stm {

Status HostAllocator::allocate(uint64_t bytes, void** ptr) {
  *ptr = std::malloc(bytes ? bytes : 1);
  return *ptr ? Status::Ok : Status::CapacityExceeded;
}
void HostAllocator::release(void* ptr) { std::free(ptr); }
Status HostAllocator::zero(void* ptr, uint64_t bytes) {
  std::memset(ptr, 0, bytes);
  return Status::Ok;
}
Status HostAllocator::copy_from_host(void* dst, const void* src, uint64_t bytes) {
  std::memcpy(dst, src, bytes);
  return Status::Ok;
}

DeviceLedger::DeviceLedger(std::string module_tag, std::shared_ptr<Allocator> alloc)
    : tag_(std::move(module_tag)), alloc_(std::move(alloc)) {
  if (!alloc_) fail(Status::InvalidArgument, tag_ + ": ledger without an allocator");
}

DeviceLedger::~DeviceLedger() { release_all(); }

void* DeviceLedger::allocate(uint64_t bytes, bool zeroed) {
  if (ptrs_.size() >= kMaxDeviceAllocations)
    fail(Status::CapacityExceeded, tag_ + ": more than 4096 device allocations");
  void* p = nullptr;
  const Status s = alloc_->allocate(bytes, &p);
  if (s != Status::Ok || !p) fail(Status::CapacityExceeded, tag_ + ": device allocation failed");
  if (zeroed && alloc_->zero(p, bytes) != Status::Ok) {
    alloc_->release(p);
    fail(Status::InternalError, tag_ + ": device clear failed");
  }
  ptrs_.push_back(p);
  sizes_.push_back(bytes);
  resident_ += bytes;
  return p;
}

void DeviceLedger::rollback(uint32_t count) {
  while (ptrs_.size() > count) {
    alloc_->release(ptrs_.back());
    resident_ -= sizes_.back();
    ptrs_.pop_back();
    sizes_.pop_back();
  }
}

void pack_read(const std::string& tag, std::FILE* f, uint64_t offset, void* dst, uint64_t bytes) {
  if (!f) fail(Status::InvalidArgument, tag + ": no pack file");
  if (std::fseek(f, (long)offset, SEEK_SET) != 0) fail(Status::IoError, tag + ": pack seek failed");
  if (bytes && std::fread(dst, 1, bytes, f) != bytes) fail(Status::IoError, tag + ": short pack read");
}

void* load_device_region(DeviceLedger& ledger, std::FILE* f, uint64_t offset, uint64_t bytes) {
  const uint32_t mark = ledger.count();
  void* dev = ledger.allocate(bytes);
  std::vector<uint8_t> chunk((size_t)std::min<uint64_t>(bytes ? bytes : 1, kStagingChunkBytes));
  try {
    for (uint64_t done = 0; done < bytes;) {
      const uint64_t n = std::min<uint64_t>(chunk.size(), bytes - done);
      pack_read(ledger.tag(), f, offset + done, chunk.data(), n);
      if (ledger.allocator().copy_from_host(static_cast<uint8_t*>(dev) + done, chunk.data(), n) != Status::Ok)
        fail(Status::InternalError, ledger.tag() + ": host->device copy failed");
      done += n;
    }
  } catch (...) {
    ledger.rollback(mark);
    throw;
  }
  return dev;
}

SlotTable::SlotTable(uint32_t slots) : states_(slots) {
  if (slots == 0) fail(Status::InvalidArgument, "slot table: no slots");
  for (auto& s : states_) s.store(kSlotFree, std::memory_order_relaxed);
}

bool SlotTable::claim(uint32_t* index) {
  for (uint32_t i = 0; i < states_.size(); ++i) {
    uint32_t expect = kSlotFree;
    if (states_[i].compare_exchange_strong(expect, kSlotClaimed, std::memory_order_acq_rel)) {
      *index = i;
      return true;
    }
  }
  return false;
}

void SlotTable::release(uint32_t index) {
  if (index >= states_.size()) fail(Status::InvalidArgument, "slot table: index out of range");
  states_[index].store(kSlotFree, std::memory_order_release);
}

Status SlotTable::claim_set(const std::vector<uint32_t>& indices) {
  for (size_t k = 0; k < indices.size(); ++k) {
    const uint32_t i = indices[k];
    uint32_t expect = kSlotFree;
    if (i >= states_.size() || !states_[i].compare_exchange_strong(expect, kSlotClaimed, std::memory_order_acq_rel)) {
      for (size_t r = 0; r < k; ++r) states_[indices[r]].store(kSlotFree, std::memory_order_release);
      return i >= states_.size() ? Status::InvalidArgument : Status::Busy;
    }
  }
  return Status::Ok;
}

void SlotTable::release_set(const std::vector<uint32_t>& indices) {
  for (uint32_t i : indices) release(i);
}

uint32_t SlotTable::free_count() const {
  uint32_t n = 0;
  for (const auto& s : states_) n += s.load(std::memory_order_acquire) == kSlotFree ? 1 : 0;
  return n;
}

bool SlotTable::claimed(uint32_t index) const {
  return index < states_.size() && states_[index].load(std::memory_order_acquire) == kSlotClaimed;
}

Status SlotTable::wait_all_free(uint64_t timeout_ns) const {
  const auto t0 = std::chrono::steady_clock::now();
  while (free_count() != states_.size()) {
    if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count() >
        timeout_ns)
      return Status::Busy;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  return Status::Ok;
}

std::string env_text(const std::string& tag, const std::string& name, const std::string& fallback) {
  const char* v = std::getenv(name.c_str());
  if (!v) return fallback;
  if (!*v) fail(Status::InvalidArgument, tag + ": " + name + " is set but empty");
  return v;
}

uint64_t env_unsigned(const std::string& tag, const std::string& name, uint64_t minimum, uint64_t maximum,
                      uint64_t fallback) {
  const char* v = std::getenv(name.c_str());
  if (!v) return fallback;
  char* end = nullptr;
  errno = 0;
  const unsigned long long x = std::strtoull(v, &end, 10);
  if (!*v || *end || errno || x < minimum || x > maximum)
    fail(Status::InvalidArgument, tag + ": " + name + " must be an integer in [" + std::to_string(minimum) + ", " +
                                      std::to_string(maximum) + "]");
  return x;
}

}  // namespace stm
}  // namespace spc
