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

// ---------------------------------------------------------------- tier mover
uint32_t state_block_equivalents(uint32_t state_bytes, uint32_t block_bytes) {
  if (!state_bytes || !block_bytes) return 0;
  return (state_bytes + block_bytes - 1) / block_bytes;
}

std::vector<uint32_t> cumulative_nonresident(const std::vector<PendingLane>& lanes,
                                             const std::vector<uint32_t>& packet_lane_counts,
                                             uint32_t state_equivalents) {
  if (lanes.empty() || packet_lane_counts.empty()) fail(Status::InvalidArgument, "tier mover: empty plan");
  uint64_t covered = 0;
  for (uint32_t n : packet_lane_counts) {
    if (n == 0) fail(Status::InvalidArgument, "tier mover: a packet without lanes");
    covered += n;
  }
  if (covered != lanes.size()) fail(Status::InvalidArgument, "tier mover: packet lane counts do not cover the lanes");
  std::vector<uint32_t> out(packet_lane_counts.size());
  uint64_t total = 0;
  auto lane = lanes.begin();
  for (size_t p = 0; p < packet_lane_counts.size(); ++p) {
    for (auto end = lane + packet_lane_counts[p]; lane != end; ++lane) {
      if (!lane->sequence) fail(Status::InvalidArgument, "tier mover: sequence id 0");
      total += lane->blocks.size() + (lane->state_nonresident ? state_equivalents : 0);
    }
    if (total > 0xffffffffull) fail(Status::CapacityExceeded, "tier mover: block count overflow");
    out[p] = uint32_t(total);
  }
  return out;
}

TierMover::TierMover(const PlanConfig& c, StageKvClient& client, const Staging& staging)
    : cfg_(c), client_(client), st_(staging) {
  if (!c.model_fp || !c.layout_fp || !c.block_bytes || !c.state_bytes)
    fail(Status::InvalidArgument, "tier mover: fingerprints and record sizes must be non-zero");
  if (!staging.blocks || !staging.states || !staging.block_records || !staging.batch_blocks)
    fail(Status::InvalidArgument, "tier mover: staging area");
}

void TierMover::set_pressure(uint32_t physical_capacity, uint32_t allocated, uint32_t staging_capacity) {
  cfg_.physical_capacity = physical_capacity;
  cfg_.allocated = allocated;
  cfg_.staging_capacity = staging_capacity;
}

uint32_t TierMover::restore_packets(const std::vector<uint32_t>& cumulative) const {
  return select_lookahead(cfg_.lookahead, uint32_t(cumulative.size()), cfg_.physical_capacity, cfg_.allocated,
                          cfg_.staging_capacity, cumulative);
}

Block TierMover::record(uint64_t sequence, uint32_t logical, uint32_t op, uint8_t* at, uint32_t bytes) const {
  Block b;
  b.op = op;
  b.key = format_key(cfg_.model_fp, cfg_.layout_fp, cfg_.rank, sequence, logical);
  b.payload = at;
  b.bytes = bytes;
  return b;
}

RestoreBatch TierMover::plan_restore(const std::vector<PendingLane>& lanes,
                                     const std::vector<uint32_t>& packet_lane_counts) const {
  if (lanes.empty()) fail(Status::InvalidArgument, "tier mover: nothing to restore");
  uint64_t covered = 0;
  for (uint32_t n : packet_lane_counts) covered += n;
  if (covered != lanes.size()) fail(Status::InvalidArgument, "tier mover: packet lane counts do not cover the lanes");
  // Prefix sums of the three resources a lane consumes; all three are monotone, so
  // the lanes that fit are a prefix whose length is the smallest of three searches.
  const size_t n = lanes.size();
  std::vector<uint64_t> recs(n + 1, 0), blks(n + 1, 0), states(n + 1, 0);
  for (size_t i = 0; i < n; ++i) {
    if (!lanes[i].sequence) fail(Status::InvalidArgument, "tier mover: sequence id 0");
    const uint32_t s = lanes[i].state_nonresident ? 1 : 0;
    blks[i + 1] = blks[i] + lanes[i].blocks.size();
    states[i + 1] = states[i] + s;
    recs[i + 1] = recs[i] + lanes[i].blocks.size() + s;
  }
  auto fitting = [](const std::vector<uint64_t>& prefix, uint64_t cap) {
    return size_t(std::upper_bound(prefix.begin() + 1, prefix.end(), cap) - (prefix.begin() + 1));
  };
  const size_t take = std::min({fitting(recs, st_.batch_blocks), fitting(blks, st_.block_records),
                                fitting(states, st_.state_records)});
  if (take == 0) fail(Status::CapacityExceeded, "tier mover: the first lane does not fit");
  RestoreBatch rb;
  rb.lanes_built = uint32_t(take);
  rb.block_records = uint32_t(blks[take]);
  rb.state_records = uint32_t(states[take]);
  rb.blocks.reserve(recs[take]);
  for (size_t i = 0; i < take; ++i) {
    const PendingLane& l = lanes[i];
    if (l.state_nonresident)
      rb.blocks.push_back(record(l.sequence, kStateBlock, Get, st_.states + states[i] * cfg_.state_bytes,
                                 cfg_.state_bytes));
    uint8_t* at = st_.blocks + blks[i] * cfg_.block_bytes;
    for (uint32_t logical : l.blocks) {
      rb.blocks.push_back(record(l.sequence, logical, Get, at, cfg_.block_bytes));
      at += cfg_.block_bytes;
    }
  }
  return rb;
}

std::vector<Block> TierMover::plan_evict(uint64_t sequence, const std::vector<uint32_t>& resident,
                                         bool include_state, const uint8_t* block_src,
                                         const uint8_t* state_src) const {
  if (!sequence) fail(Status::InvalidArgument, "tier mover: sequence id 0");
  const size_t n = resident.size() + (include_state ? 1 : 0);
  if (n == 0) fail(Status::InvalidArgument, "tier mover: nothing to evict");
  if (n > st_.batch_blocks) fail(Status::CapacityExceeded, "tier mover: evict batch too large");
  if ((!resident.empty() && !block_src) || (include_state && !state_src))
    fail(Status::InvalidArgument, "tier mover: evict source");
  std::vector<Block> out;
  out.reserve(n);
  if (include_state)
    out.push_back(record(sequence, kStateBlock, Put, const_cast<uint8_t*>(state_src), cfg_.state_bytes));
  for (size_t i = 0; i < resident.size(); ++i)
    out.push_back(record(sequence, resident[i], Put, const_cast<uint8_t*>(block_src) + i * cfg_.block_bytes,
                         cfg_.block_bytes));
  return out;
}

void TierMover::start(Direction d, const std::vector<Block>& blocks, uint32_t priority) {
  if (priority > kPrioritySpeculative) fail(Status::InvalidArgument, "tier mover: priority");
  Channel& ch = ch_[uint32_t(d)];
  if (ch.stage != Free) fail(Status::InvalidArgument, "tier mover: the channel already carries a batch");
  const uint32_t op = d == Direction::Restore ? Get : Put;
  ch.batch_id = client_.submit(op, blocks, priority);
  ch.blocks = uint32_t(blocks.size());
  ch.outcome = Status::Pending;
  ch.stage = InFlight;
}

void TierMover::poll() {
  for (Channel& ch : ch_) {
    if (ch.stage != InFlight) continue;
    Completion done;
    const Status s = client_.poll(ch.batch_id, done);
    if (s == Status::Pending || s == Status::Busy) continue;
    if (s != Status::Ok) fail(s, "tier mover: poll failed");
    if (done.batch_id != ch.batch_id || done.completed_blocks > ch.blocks)
      fail(Status::AbiMismatch, "tier mover: completion does not match the batch");
    ch.outcome = done.status;
    ch.stage = Landed;
  }
}

Status TierMover::collect(Direction d) {
  Channel& ch = ch_[uint32_t(d)];
  if (ch.stage != Landed) fail(Status::InvalidArgument, "tier mover: no landed batch to collect");
  const Status s = ch.outcome;
  ch = Channel{};
  return s;
}

}  // namespace kvt
}  // namespace spc
