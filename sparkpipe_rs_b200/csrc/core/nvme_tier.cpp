#include "nvme_tier.h"

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>

namespace spc {
namespace nvt {

// ---------------------------------------------------------------- file device
FileDevice::FileDevice(const std::string& path, uint64_t size_bytes, uint32_t threads) {
#ifdef O_DIRECT
  fd_ = ::open(path.c_str(), O_RDWR | O_CREAT | O_DIRECT, 0644);
  direct_ = fd_ >= 0;
#endif
  if (fd_ < 0) fd_ = ::open(path.c_str(), O_RDWR | O_CREAT, 0644);
  if (fd_ < 0) fail(Status::IoError, "nvme tier: cannot open " + path + ": " + std::strerror(errno));
  if (size_bytes && ::ftruncate(fd_, (off_t)size_bytes) != 0) {
    ::close(fd_);
    fail(Status::IoError, "nvme tier: cannot size " + path);
  }
  for (uint32_t i = 0; i < std::max<uint32_t>(1, threads); ++i) workers_.emplace_back([this] { worker(); });
}

FileDevice::~FileDevice() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : workers_) t.join();
  if (fd_ >= 0) ::close(fd_);
}

static bool aligned(uint64_t v) { return v % kIoAlignment == 0; }

Status FileDevice::submit_read(uint64_t offset, void* dst, uint32_t bytes, uint64_t* ticket) {
  if (direct_ && !(aligned(offset) && aligned(bytes) && aligned(reinterpret_cast<uintptr_t>(dst))))
    return Status::InvalidArgument;
  std::lock_guard<std::mutex> g(mu_);
  *ticket = next_ticket_++;
  queue_.push_back(Req{*ticket, offset, dst, bytes});
  cv_.notify_one();
  return Status::Ok;
}

void FileDevice::worker() {
  while (true) {
    Req r;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
      if (queue_.empty()) return;  // stopping with nothing queued
      r = queue_.front();
      queue_.pop_front();
    }
    Status st = Status::Ok;
    uint32_t got = 0;
    while (got < r.bytes) {
      const ssize_t n = ::pread(fd_, static_cast<uint8_t*>(r.dst) + got, r.bytes - got, (off_t)(r.offset + got));
      if (n < 0 && errno == EINTR) continue;
      if (n < 0) { st = Status::IoError; break; }
      if (n == 0) {  // past the end of the file: never written, reads as zeros
        std::memset(static_cast<uint8_t*>(r.dst) + got, 0, r.bytes - got);
        break;
      }
      got += (uint32_t)n;
    }
    std::lock_guard<std::mutex> g(mu_);
    done_[r.ticket] = st;
  }
}

Status FileDevice::poll(uint64_t ticket) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = done_.find(ticket);
  if (it != done_.end()) {
    const Status s = it->second;
    done_.erase(it);
    return s;
  }
  return ticket < next_ticket_ ? Status::Busy : Status::NotFound;
}

Status FileDevice::write(uint64_t offset, const void* src, uint32_t bytes) {
  if (direct_ && !(aligned(offset) && aligned(bytes) && aligned(reinterpret_cast<uintptr_t>(src))))
    return Status::InvalidArgument;
  uint32_t put = 0;
  while (put < bytes) {
    const ssize_t n = ::pwrite(fd_, static_cast<const uint8_t*>(src) + put, bytes - put, (off_t)(offset + put));
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) return Status::IoError;
    put += (uint32_t)n;
  }
  return Status::Ok;
}

// ---------------------------------------------------------------- mock device
MockDevice::MockDevice(uint64_t size_bytes, uint32_t latency_polls) : mem_(size_bytes, 0), latency_(latency_polls) {}

Status MockDevice::submit_read(uint64_t offset, void* dst, uint32_t bytes, uint64_t* ticket) {
  if (offset + bytes > mem_.size()) return Status::InvalidArgument;
  *ticket = next_ticket_++;
  live_[*ticket] = Req{offset, dst, bytes, latency_, fail_next_};
  fail_next_ = false;
  ++reads_;
  return Status::Ok;
}

Status MockDevice::poll(uint64_t ticket) {
  auto it = live_.find(ticket);
  if (it == live_.end()) return Status::NotFound;
  Req& r = it->second;
  if (r.polls_left > 0) {
    --r.polls_left;
    return Status::Busy;
  }
  const Status s = r.fail ? Status::IoError : Status::Ok;
  if (!r.fail) std::memcpy(r.dst, mem_.data() + r.offset, r.bytes);
  live_.erase(it);
  return s;
}

Status MockDevice::cancel(uint64_t ticket) {
  live_.erase(ticket);
  return Status::Ok;
}

Status MockDevice::write(uint64_t offset, const void* src, uint32_t bytes) {
  if (offset + bytes > mem_.size()) return Status::InvalidArgument;
  std::memcpy(mem_.data() + offset, src, bytes);
  return Status::Ok;
}

// ---------------------------------------------------------------- tier
Tier::Tier(const Config& cfg, std::shared_ptr<BlockDevice> device) : cfg_(cfg), dev_(std::move(device)) {
  if (!dev_) fail(Status::InvalidArgument, "nvme tier: no device");
  if (cfg.block_bytes == 0 || cfg.block_bytes % kIoAlignment)
    fail(Status::InvalidArgument, "nvme tier: block bytes must be a positive multiple of 4096");
  if (cfg.staging_buffers < 2 || cfg.staging_buffers > kMaxStagingBuffers || cfg.demand_reserve >= cfg.staging_buffers)
    fail(Status::InvalidArgument, "nvme tier: 2..16 staging buffers, fewer reserved for demand");
  if (cfg.pending_capacity == 0 || cfg.budget_bytes < cfg.block_bytes || cfg.device_bytes_per_second == 0 ||
      cfg.step_microseconds == 0 || cfg.base_offset % kIoAlignment)
    fail(Status::InvalidArgument, "nvme tier: invalid configuration");
  const uint64_t n = cfg.budget_bytes / cfg.block_bytes;
  if (n > (1ull << 26)) fail(Status::InvalidArgument, "nvme tier: more than 2^26 slots; use larger blocks");
  slots_.resize(n);
  free_.reserve(n);
  for (uint64_t i = n; i-- > 0;) free_.push_back((uint32_t)i);
  bufs_.resize(cfg.staging_buffers);
  staging_ = static_cast<uint8_t*>(std::aligned_alloc(kIoAlignment, (size_t)cfg.staging_buffers * cfg.block_bytes));
  if (!staging_) fail(Status::CapacityExceeded, "nvme tier: staging allocation failed");
  const double bytes_per_step = double(cfg.device_bytes_per_second) * cfg.step_microseconds * 1e-6;
  transfer_steps_ = std::max<uint32_t>(1, (uint32_t)std::ceil(cfg.block_bytes / std::max(1.0, bytes_per_step)));
  stats_.slot_count = n;
}

Tier::~Tier() {
  drain(1u << 30);
  std::free(staging_);
}

uint32_t Tier::inflight() const {
  uint32_t n = 0;
  for (const auto& b : bufs_) n += b.state == Reading ? 1 : 0;
  return n;
}

uint32_t Tier::drain(uint32_t max_polls) {
  for (uint32_t it = 0; it < max_polls && inflight() > 0; ++it) {
    for (auto& b : bufs_) {
      if (b.state != Reading) continue;
      const Status s = dev_->poll(b.ticket);
      if (s != Status::Busy) b = Buffer{};
    }
    if (inflight() > 0) std::this_thread::yield();
  }
  return inflight();
}

uint32_t Tier::evict_one() {
  const uint32_t n = (uint32_t)slots_.size();
  for (uint64_t step = 0; step < 2ull * n; ++step) {
    const uint32_t s = hand_;
    hand_ = (hand_ + 1) % n;
    Slot& sl = slots_[s];
    if (sl.state != Committed) continue;
    if (sl.pins > 0) {
      ++stats_.pinned_skips;
      continue;
    }
    if (sl.referenced) {
      sl.referenced = false;
      continue;
    }
    index_.erase(sl.hash);
    sl = Slot{0, sl.generation + 1, Free, false, 0};
    ++stats_.evictions;
    --stats_.slots_in_use;
    return s;
  }
  return UINT32_MAX;
}

Reservation Tier::reserve_write(uint64_t hash) {
  ++stats_.write_reservations;
  Reservation r;
  r.hash = hash;
  auto it = index_.find(hash);
  if (it != index_.end()) {
    r.slot = it->second;
    r.generation = slots_[r.slot].generation;
    r.offset = cfg_.base_offset + uint64_t(r.slot) * cfg_.block_bytes;
    r.already_present = true;
    slots_[r.slot].referenced = true;
    return r;
  }
  uint32_t s;
  if (!free_.empty()) {
    s = free_.back();
    free_.pop_back();
  } else {
    s = evict_one();
    if (s == UINT32_MAX) fail(Status::CapacityExceeded, "nvme tier: every slot is pinned or reserved");
  }
  Slot& sl = slots_[s];
  sl.hash = hash;
  sl.state = Reserved;
  sl.referenced = false;
  sl.pins = 0;
  ++stats_.slots_in_use;
  r.slot = s;
  r.generation = sl.generation;
  r.offset = cfg_.base_offset + uint64_t(s) * cfg_.block_bytes;
  return r;
}

void Tier::commit_write(const Reservation& r) {
  if (r.already_present) return;
  if (r.slot >= slots_.size()) fail(Status::InvalidArgument, "nvme tier: bad reservation");
  Slot& sl = slots_[r.slot];
  if (sl.state != Reserved || sl.generation != r.generation || sl.hash != r.hash)
    fail(Status::InvalidArgument, "nvme tier: reservation no longer held");
  sl.state = Committed;
  sl.referenced = true;
  index_[r.hash] = r.slot;
  ++stats_.publishes;
}

void Tier::abort_write(const Reservation& r) {
  if (r.already_present) return;
  if (r.slot >= slots_.size()) fail(Status::InvalidArgument, "nvme tier: bad reservation");
  Slot& sl = slots_[r.slot];
  if (sl.state != Reserved || sl.generation != r.generation || sl.hash != r.hash)
    fail(Status::InvalidArgument, "nvme tier: reservation no longer held");
  sl = Slot{0, sl.generation + 1, Free, false, 0};
  free_.push_back(r.slot);
  --stats_.slots_in_use;
  ++stats_.write_aborts;
}

bool Tier::offset_of(uint64_t hash, uint64_t* offset) const {
  auto it = index_.find(hash);
  if (it == index_.end()) return false;
  *offset = cfg_.base_offset + uint64_t(it->second) * cfg_.block_bytes;
  return true;
}

int Tier::buffer_of(uint64_t hash) const {
  for (size_t b = 0; b < bufs_.size(); ++b)
    if (bufs_[b].state != Idle && !bufs_[b].cancelling && bufs_[b].hash == hash) return (int)b;
  return -1;
}

int Tier::free_buffer(bool for_demand) {
  uint32_t idle = 0;
  int first = -1;
  for (size_t b = 0; b < bufs_.size(); ++b)
    if (bufs_[b].state == Idle) {
      ++idle;
      if (first < 0) first = (int)b;
    }
  if (first >= 0 && (for_demand || idle > cfg_.demand_reserve)) return first;
  if (!for_demand) return -1;
  auto pinned = [&](const Buffer& b) {
    auto it = index_.find(b.hash);
    return it != index_.end() && slots_[it->second].pins > 0;
  };
  // a demand may take a landed, unconsumed prefetch first, then an in-flight one
  for (size_t b = 0; b < bufs_.size(); ++b) {
    Buffer& x = bufs_[b];
    if (x.state == Ready && !x.demand && !pinned(x)) {
      x = Buffer{};
      ++stats_.prefetch_dropped;
      ++stats_.prefetch_preemptions;
      return (int)b;
    }
  }
  for (size_t b = 0; b < bufs_.size(); ++b) {
    Buffer& x = bufs_[b];
    if (x.state == Reading && !x.demand && !x.cancelling && !pinned(x)) {
      if (dev_->cancel(x.ticket) == Status::Ok) {
        x = Buffer{};
        ++stats_.prefetch_preemptions;
        return (int)b;
      }
      x.cancelling = true;  // device-owned until its read ends; pump reclaims it
      ++stats_.prefetch_preemptions;
    }
  }
  return -1;
}

bool Tier::issue(int b, uint32_t slot, bool demand, uint32_t step_now, uint32_t need_by) {
  Buffer& x = bufs_[b];
  uint64_t ticket = 0;
  const uint64_t off = cfg_.base_offset + uint64_t(slot) * cfg_.block_bytes;
  if (dev_->submit_read(off, staging_ + size_t(b) * cfg_.block_bytes, cfg_.block_bytes, &ticket) != Status::Ok) {
    ++stats_.io_errors;
    return false;
  }
  x.state = Reading;
  x.demand = demand;
  x.cancelling = false;
  x.hash = slots_[slot].hash;
  x.slot = slot;
  x.generation = slots_[slot].generation;
  x.ticket = ticket;
  x.issued_step = step_now;
  x.need_by = need_by;
  stats_.read_bytes += cfg_.block_bytes;
  return true;
}

PlanReport Tier::plan_lookahead(const std::vector<Need>& needs, uint32_t step_now) {
  PlanReport rep;
  for (const Need& n : needs) {
    const int b = buffer_of(n.hash);
    if (b >= 0) {
      Buffer& x = bufs_[b];
      x.need_by = std::min(x.need_by, n.need_by_step);
      if (x.state == Ready) ++rep.ready;
      else ++rep.inflight;
      continue;
    }
    auto it = index_.find(n.hash);
    if (it == index_.end()) {
      ++rep.absent;
      continue;
    }
    slots_[it->second].referenced = true;
    auto pit = std::find_if(pending_.begin(), pending_.end(), [&](const Pending& p) { return p.hash == n.hash; });
    if (pit != pending_.end()) {
      if (n.need_by_step < pit->need_by) {
        pending_.erase(pit);
      } else {
        ++rep.queued;
        continue;
      }
    } else if (pending_.size() >= cfg_.pending_capacity) {
      ++rep.queue_full;
      continue;
    }
    auto pos = std::upper_bound(pending_.begin(), pending_.end(), n.need_by_step,
                                [](uint32_t v, const Pending& p) { return v < p.need_by; });
    pending_.insert(pos, Pending{n.hash, n.need_by_step, false});
    ++rep.queued;
    if (n.need_by_step < step_now + transfer_steps_) ++rep.late_risk;
  }
  return rep;
}

Demand Tier::request_demand(uint64_t hash, uint32_t step_now, const uint8_t** staging) {
  *staging = nullptr;
  const int b = buffer_of(hash);
  if (b >= 0) {
    Buffer& x = bufs_[b];
    x.demand = true;
    if (x.state == Ready) {
      *staging = staging_ + size_t(b) * cfg_.block_bytes;
      ++stats_.demand_hits;
      return Demand::Ready;
    }
    ++stats_.demand_joins;
    return Demand::InFlight;
  }
  auto it = index_.find(hash);
  if (it == index_.end()) {
    ++stats_.demand_misses;
    return Demand::Miss;
  }
  pending_.erase(std::remove_if(pending_.begin(), pending_.end(), [&](const Pending& p) { return p.hash == hash; }),
                 pending_.end());
  slots_[it->second].referenced = true;
  const int fb = free_buffer(true);
  if (fb < 0) {  // every staging buffer holds demand data: a sizing error; retry from the queue head
    ++stats_.demand_stalls;
    pending_.insert(pending_.begin(), Pending{hash, step_now, true});
    return Demand::InFlight;
  }
  if (!issue(fb, it->second, true, step_now, step_now)) {
    ++stats_.demand_misses;
    return Demand::Miss;
  }
  ++stats_.demand_loads;
  return Demand::Started;
}

void Tier::pump(uint32_t step_now) {
  for (auto& x : bufs_) {
    if (x.state != Reading) continue;
    const Status s = dev_->poll(x.ticket);
    if (s == Status::Busy) continue;
    if (x.cancelling) {  // a cancelled read that finally ended
      x = Buffer{};
      continue;
    }
    if (s != Status::Ok) {
      ++stats_.io_errors;
      x = Buffer{};
      continue;
    }
    const Slot& sl = slots_[x.slot];
    if (sl.state != Committed || sl.generation != x.generation || sl.hash != x.hash) {
      ++stats_.stale_completions;  // the slot was evicted while the read ran
      x = Buffer{};
      continue;
    }
    x.state = Ready;
    if (!x.demand) {
      ++stats_.prefetch_landings;
      if (step_now > x.need_by) ++stats_.prefetch_late;
    }
  }
  while (!pending_.empty()) {
    const Pending p = pending_.front();
    auto it = index_.find(p.hash);
    if (it == index_.end() || buffer_of(p.hash) >= 0) {  // evicted meanwhile, or already moving
      pending_.erase(pending_.begin());
      continue;
    }
    const int b = free_buffer(p.demand);
    if (b < 0) break;
    pending_.erase(pending_.begin());
    if (issue(b, it->second, p.demand, step_now, p.need_by)) ++(p.demand ? stats_.demand_loads : stats_.prefetch_issues);
  }
}

bool Tier::consume(uint64_t hash) {
  const int b = buffer_of(hash);
  if (b < 0 || bufs_[b].state != Ready) return false;
  bufs_[b] = Buffer{};
  return true;
}

bool Tier::pin(uint64_t hash, bool on) {
  auto it = index_.find(hash);
  if (it == index_.end()) return false;
  Slot& sl = slots_[it->second];
  sl.pins = on ? sl.pins + 1 : std::max(0, sl.pins - 1);
  return true;
}

Residency Tier::will_be_resident_by(const std::vector<uint64_t>& hashes, uint32_t step_now,
                                    uint32_t step_deadline) const {
  Residency r;
  const uint32_t lanes = std::max<uint32_t>(1, cfg_.staging_buffers - cfg_.demand_reserve);
  for (uint64_t h : hashes) {
    const int b = buffer_of(h);
    if (b >= 0) {
      const Buffer& x = bufs_[b];
      if (x.state == Ready) ++r.ready;
      else if (x.issued_step + transfer_steps_ <= step_deadline) ++r.inflight_on_time;
      else ++r.late;
      continue;
    }
    if (!index_.count(h)) {
      ++r.absent;
      continue;
    }
    // queued reads ahead of it share the prefetch lanes
    uint32_t ahead = 0;
    for (const Pending& p : pending_) {
      if (p.hash == h) break;
      ++ahead;
    }
    const uint32_t eta = step_now + transfer_steps_ * (1 + ahead / lanes);
    if (eta <= step_deadline) ++r.planned_on_time;
    else ++r.late;
  }
  const uint32_t good = r.ready + r.inflight_on_time + r.planned_on_time;
  r.confidence = (r.late == 0 && r.absent == 0) ? Confidence::All : (good == 0 ? Confidence::None : Confidence::Partial);
  return r;
}

}  // namespace nvt
}  // namespace spc
