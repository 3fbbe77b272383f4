#include "kv_tier.h"

#include <algorithm>
#include <cstdio>
#include <cstring>

namespace spc {
namespace kvt {

std::string format_key(uint64_t model_fp, uint64_t layout_fp, uint32_t rank, uint64_t sequence, uint32_t block) {
  char buf[kMaxKeyBytes];
  int n;
  if (block == kStateBlock)
    n = std::snprintf(buf, sizeof buf, "sp/m%016llx/c%016llx/r%u/s%llu/state", (unsigned long long)model_fp,
                      (unsigned long long)layout_fp, rank, (unsigned long long)sequence);
  else
    n = std::snprintf(buf, sizeof buf, "sp/m%016llx/c%016llx/r%u/s%llu/b%u", (unsigned long long)model_fp,
                      (unsigned long long)layout_fp, rank, (unsigned long long)sequence, block);
  if (n < 0 || n >= int(kMaxKeyBytes)) fail(Status::CapacityExceeded, "kv tier: key too long");
  return std::string(buf, size_t(n));
}

uint32_t normalize_lookahead(uint32_t lookahead, uint32_t queue_depth) {
  uint32_t n = lookahead == 0 ? kDefaultLookahead : lookahead;
  n = std::min(n, kMaxLookahead);
  return std::min(n, queue_depth);
}

uint32_t select_lookahead(uint32_t lookahead, uint32_t queue_depth, uint32_t physical_capacity, uint32_t allocated,
                          uint32_t staging_capacity, const std::vector<uint32_t>& cumulative) {
  const uint32_t n = normalize_lookahead(lookahead, std::min<uint32_t>(queue_depth, uint32_t(cumulative.size())));
  const uint32_t free_blocks = physical_capacity > allocated ? physical_capacity - allocated : 0;
  const uint32_t room = std::min(free_blocks, staging_capacity);
  uint32_t take = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if (cumulative[i] > room) break;
    take = i + 1;
  }
  return take;
}

// ---------------------------------------------------------------- memory store
MemoryStore::MemoryStore() : worker_([this] { run(); }) {}

MemoryStore::~MemoryStore() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  worker_.join();
}

Status MemoryStore::submit(uint64_t batch_id, const std::vector<Block>& blocks, uint32_t) {
  std::lock_guard<std::mutex> lk(mu_);
  if (known_.count(batch_id)) return Status::Duplicate;
  known_[batch_id] = true;
  queue_.push_back(Job{batch_id, blocks});
  cv_.notify_all();
  return Status::Ok;
}

Status MemoryStore::poll(uint64_t batch_id, Completion& out) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = done_.find(batch_id);
  if (it != done_.end()) {
    out = it->second;
    done_.erase(it);
    known_.erase(batch_id);
    return Status::Ok;
  }
  return known_.count(batch_id) ? Status::Pending : Status::NotFound;
}

size_t MemoryStore::stored_blocks() const {
  std::lock_guard<std::mutex> lk(mu_);
  return data_.size();
}

void MemoryStore::set_paused(bool paused) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    paused_ = paused;
  }
  cv_.notify_all();
}

void MemoryStore::run() {
  std::unique_lock<std::mutex> lk(mu_);
  while (true) {
    cv_.wait(lk, [this] { return stop_ || (!paused_ && !queue_.empty()); });
    if (stop_) return;
    Job job = std::move(queue_.front());
    queue_.pop_front();
    Completion c;
    c.batch_id = job.id;
    c.status = Status::Ok;
    for (const Block& b : job.blocks) {
      if (b.op == Put) {
        data_[b.key].assign(b.payload, b.payload + b.bytes);
      } else {
        auto it = data_.find(b.key);
        if (it == data_.end() || it->second.size() != b.bytes) {
          c.status = Status::NotFound;  // a restore of a block that was never stored
          break;
        }
        std::memcpy(b.payload, it->second.data(), b.bytes);
      }
      ++c.completed_blocks;
    }
    done_[job.id] = c;
  }
}

// ---------------------------------------------------------------- stage client
StageKvClient::StageKvClient(const std::string& provider, std::shared_ptr<Store> store, uint32_t rank,
                             uint64_t model_fp, uint64_t layout_fp)
    : enabled_(provider != "none"), store_(std::move(store)), rank_(rank), model_fp_(model_fp), layout_fp_(layout_fp) {
  if (provider.empty()) fail(Status::InvalidArgument, "kv tier: the provider must be named (or \"none\")");
  if (enabled_ && !store_) fail(Status::InvalidArgument, "kv tier: an enabled tier needs a store");
  if (model_fp == 0 || layout_fp == 0) fail(Status::InvalidArgument, "kv tier: fingerprints must be non-zero");
}

uint64_t StageKvClient::submit(uint32_t op, const std::vector<Block>& blocks, uint32_t priority) {
  if (!enabled_) fail(Status::NotFound, "kv tier: disabled");
  if (op != Get && op != Put) fail(Status::InvalidArgument, "kv tier: operation");
  if (blocks.empty() || blocks.size() > kMaxBatchBlocks) fail(Status::InvalidArgument, "kv tier: batch size");
  if (inflight_.size() >= kMaxInflightBatches) fail(Status::Busy, "kv tier: too many batches in flight");
  for (const Block& b : blocks)
    if (b.op != op || !b.payload || !b.bytes || b.key.empty() || b.key.size() >= kMaxKeyBytes)
      fail(Status::InvalidArgument, "kv tier: malformed block");
  const uint64_t id = next_id_++;
  const Status s = store_->submit(id, blocks, priority);
  if (s != Status::Ok) fail(s, "kv tier: store refused the batch");
  inflight_[id] = true;
  return id;
}

Status StageKvClient::poll(uint64_t batch_id, Completion& out) {
  if (!enabled_) return Status::NotFound;
  const Status s = store_->poll(batch_id, out);
  if (s == Status::Ok) inflight_.erase(batch_id);
  return s;
}

// ---------------------------------------------------------------- work control
static void check_plan(const PlanConfig& c) {
  if (!c.model_fp || !c.layout_fp || !c.block_bytes || !c.state_bytes)
    fail(Status::InvalidArgument, "work control: fingerprints and record sizes must be non-zero");
}

static Block make_block(const PlanConfig& c, uint64_t seq, uint32_t logical, uint32_t op, uint8_t* payload,
                        uint32_t bytes) {
  if (!seq || !payload || !bytes) fail(Status::InvalidArgument, "work control: block");
  Block b;
  b.op = op;
  b.key = format_key(c.model_fp, c.layout_fp, c.rank, seq, logical);
  b.payload = payload;
  b.bytes = bytes;
  return b;
}

uint32_t state_block_equivalents(uint32_t state_bytes, uint32_t block_bytes) {
  if (!state_bytes || !block_bytes) return 0;
  return (state_bytes + block_bytes - 1) / block_bytes;
}

std::vector<uint32_t> cumulative_nonresident(const std::vector<PendingLane>& lanes,
                                             const std::vector<uint32_t>& packet_lane_counts,
                                             uint32_t state_equivalents) {
  if (lanes.empty() || packet_lane_counts.empty()) fail(Status::InvalidArgument, "work control: empty plan");
  std::vector<uint32_t> out;
  uint64_t total = 0;
  size_t li = 0;
  for (uint32_t n : packet_lane_counts) {
    if (n == 0 || n > lanes.size() - li) fail(Status::InvalidArgument, "work control: packet lane counts");
    for (uint32_t k = 0; k < n; ++k) {
      const PendingLane& l = lanes[li++];
      if (!l.sequence) fail(Status::InvalidArgument, "work control: sequence id 0");
      total += l.blocks.size() + (l.state_nonresident ? state_equivalents : 0);
      if (total > 0xffffffffull) fail(Status::CapacityExceeded, "work control: block count overflow");
    }
    out.push_back(uint32_t(total));
  }
  if (li != lanes.size()) fail(Status::InvalidArgument, "work control: lanes not covered by packets");
  return out;
}

uint32_t select_restore_packets(const PlanConfig& c, const std::vector<uint32_t>& cumulative) {
  return select_lookahead(c.lookahead, uint32_t(cumulative.size()), c.physical_capacity, c.allocated,
                          c.staging_capacity, cumulative);
}

RestoreBatch build_restore_batch(const PlanConfig& c, const std::vector<PendingLane>& lanes,
                                 const std::vector<uint32_t>& packet_lane_counts, uint8_t* block_staging,
                                 uint32_t block_staging_records, uint8_t* state_staging,
                                 uint32_t state_staging_records, uint32_t block_capacity) {
  check_plan(c);
  if (lanes.empty() || !block_staging || !state_staging || !block_capacity)
    fail(Status::InvalidArgument, "work control: restore inputs");
  uint64_t declared = 0;
  for (uint32_t n : packet_lane_counts) declared += n;
  if (declared != lanes.size()) fail(Status::InvalidArgument, "work control: packet lane counts");
  RestoreBatch rb;
  for (const PendingLane& l : lanes) {
    if (!l.sequence) fail(Status::InvalidArgument, "work control: sequence id 0");
    const uint32_t need = uint32_t(l.blocks.size()) + (l.state_nonresident ? 1 : 0);
    const bool fits = need <= block_capacity - rb.blocks.size() &&
                      l.blocks.size() <= block_staging_records - rb.block_records &&
                      (!l.state_nonresident || rb.state_records < state_staging_records);
    if (!fits) {
      if (rb.lanes_built == 0) fail(Status::CapacityExceeded, "work control: the first lane does not fit");
      break;
    }
    if (l.state_nonresident) {
      rb.blocks.push_back(make_block(c, l.sequence, kStateBlock, Get,
                                     state_staging + uint64_t(rb.state_records) * c.state_bytes, c.state_bytes));
      ++rb.state_records;
    }
    for (uint32_t blk : l.blocks) {
      rb.blocks.push_back(make_block(c, l.sequence, blk, Get,
                                     block_staging + uint64_t(rb.block_records) * c.block_bytes, c.block_bytes));
      ++rb.block_records;
    }
    ++rb.lanes_built;
  }
  return rb;
}

std::vector<Block> build_evict_batch(const PlanConfig& c, uint64_t sequence, const std::vector<uint32_t>& resident,
                                     bool include_state, uint8_t* block_staging, uint8_t* state_staging,
                                     uint32_t block_capacity) {
  check_plan(c);
  if (!sequence || !block_staging || !state_staging) fail(Status::InvalidArgument, "work control: evict inputs");
  const uint32_t n = uint32_t(resident.size()) + (include_state ? 1 : 0);
  if (n == 0) fail(Status::InvalidArgument, "work control: nothing to evict");
  if (n > block_capacity) fail(Status::CapacityExceeded, "work control: evict batch too large");
  std::vector<Block> out;
  if (include_state) out.push_back(make_block(c, sequence, kStateBlock, Put, state_staging, c.state_bytes));
  for (size_t i = 0; i < resident.size(); ++i)
    out.push_back(make_block(c, sequence, resident[i], Put, block_staging + i * c.block_bytes, c.block_bytes));
  return out;
}

void submit_batch(StageKvClient& client, BatchState& state, uint32_t op, const std::vector<Block>& blocks,
                  uint32_t priority) {
  if (priority > kPrioritySpeculative) fail(Status::InvalidArgument, "work control: priority");
  if (state.phase != Idle) fail(Status::InvalidArgument, "work control: a batch is already outstanding");
  state.batch_id = client.submit(op, blocks, priority);
  state.status = Status::Pending;
  state.phase = Submitted;
  state.submitted_blocks = uint32_t(blocks.size());
}

static void progress_one(StageKvClient& client, BatchState& s) {
  if (s.phase != Submitted) return;
  Completion c;
  const Status st = client.poll(s.batch_id, c);
  if (st == Status::Pending || st == Status::Busy) return;
  if (st != Status::Ok) fail(st, "work control: poll failed");
  if (c.batch_id != s.batch_id || c.completed_blocks > s.submitted_blocks)
    fail(Status::AbiMismatch, "work control: completion does not match the batch");
  s.status = c.status;
  s.phase = Ready;
}

void progress(StageKvClient& client, BatchState& restore, BatchState& evict) {
  progress_one(client, restore);
  progress_one(client, evict);
}

void acknowledge(BatchState& state) {
  if (state.phase != Ready) fail(Status::InvalidArgument, "work control: nothing to acknowledge");
  state = BatchState{};
}

}  // namespace kvt
}  // namespace spc
