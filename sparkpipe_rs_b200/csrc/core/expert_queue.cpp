#include "expert_queue.h"

#include <algorithm>

namespace spc {
namespace eq {

ExpertQueue::ExpertQueue(const Config& c) : cfg_(c) {
  if (c.layer_count == 0 || c.layer_count > kMaxLayers) fail(Status::InvalidArgument, "expert queue: layer count");
  if (c.expert_count == 0 || c.expert_count > kMaxExperts) fail(Status::InvalidArgument, "expert queue: expert count");
  if (c.firing_threshold_rows == 0 || c.firing_threshold_rows > kMaxFiringRows)
    fail(Status::InvalidArgument, "expert queue: firing threshold must be 1..1024 rows");
  if (c.firing_deadline_ns == 0) fail(Status::InvalidArgument, "expert queue: firing deadline must be positive");
  if (c.mode != Mode::LowLatency && c.mode != Mode::SealedBatch) fail(Status::InvalidArgument, "expert queue: mode");
  slots_.resize(size_t(c.layer_count) * c.expert_count);
  layer_rows_.assign(c.layer_count, 0);
  sealed_.assign(c.layer_count, 0);
}

uint32_t ExpertQueue::take_node() {
  if (free_ != kNil) {
    const uint32_t i = free_;
    free_ = pool_[i].next;
    return i;
  }
  if (used_high_ >= kMaxRows) return kNil;
  if (used_high_ >= pool_.size()) pool_.resize(std::min<size_t>(kMaxRows, std::max<size_t>(1024, pool_.size() * 2)));
  return used_high_++;
}

void ExpertQueue::enqueue(uint32_t layer, uint32_t expert, uint64_t row_id, uint64_t arrival_ns) {
  if (layer >= cfg_.layer_count || expert >= cfg_.expert_count) fail(Status::InvalidArgument, "expert queue: index");
  if (cfg_.mode == Mode::SealedBatch && sealed_[layer]) fail(Status::Busy, "expert queue: layer is sealed");
  const uint32_t n = take_node();
  if (n == kNil) fail(Status::CapacityExceeded, "expert queue: row pool exhausted");
  pool_[n] = Node{row_id, arrival_ns, kNil};
  Slot& s = slot(layer, expert);
  if (s.count == 0) {
    s.head = n;
    s.oldest_ns = arrival_ns;
  } else {
    pool_[s.tail].next = n;
  }
  s.tail = n;
  ++s.count;
  ++st_.enqueued;
  ++layer_rows_[layer];
}

void ExpertQueue::seal(uint32_t layer) {
  if (layer >= cfg_.layer_count) fail(Status::InvalidArgument, "expert queue: layer");
  if (cfg_.mode != Mode::SealedBatch) fail(Status::Unsupported, "expert queue: sealing needs the sealed-batch mode");
  if (sealed_[layer]) fail(Status::Busy, "expert queue: layer already sealed");
  if (layer_rows_[layer] == 0) fail(Status::NotFound, "expert queue: nothing to seal");
  for (uint32_t e = 0; e < cfg_.expert_count; ++e)
    if (slot(layer, e).count > kMaxFiringRows) fail(Status::CapacityExceeded, "expert queue: slot exceeds a firing");
  sealed_[layer] = 1;
}

void ExpertQueue::set_firing_threshold(uint32_t rows) {
  if (rows == 0 || rows > kMaxFiringRows) fail(Status::InvalidArgument, "expert queue: firing threshold");
  cfg_.firing_threshold_rows = rows;
}

bool ExpertQueue::due(uint32_t layer, const Slot& s, uint64_t now_ns) const {
  if (s.count == 0) return false;
  if (cfg_.mode == Mode::SealedBatch) return sealed_[layer] != 0;
  if (s.count >= cfg_.firing_threshold_rows) return true;
  return now_ns >= s.oldest_ns && now_ns - s.oldest_ns >= cfg_.firing_deadline_ns;
}

bool ExpertQueue::next_firing(uint64_t now_ns, Firing& out) {
  for (uint32_t l = 0; l < cfg_.layer_count; ++l) {
    if (cfg_.mode == Mode::SealedBatch && !sealed_[l]) continue;
    for (uint32_t e = 0; e < cfg_.expert_count; ++e) {
      Slot& s = slot(l, e);
      if (!due(l, s, now_ns)) continue;
      const uint32_t take = cfg_.mode == Mode::SealedBatch ? s.count : std::min(s.count, kMaxFiringRows);
      out.layer = l;
      out.expert = e;
      out.row_ids.clear();
      out.row_ids.reserve(take);
      uint32_t n = s.head;
      for (uint32_t i = 0; i < take; ++i) {
        const uint32_t next = pool_[n].next;
        out.row_ids.push_back(pool_[n].row_id);
        pool_[n].next = free_;  // back to the free list
        free_ = n;
        n = next;
      }
      s.head = n;
      if (n == kNil) s.tail = kNil;
      s.count -= take;
      if (s.count) s.oldest_ns = pool_[s.head].arrival_ns;
      st_.enqueued -= take;
      layer_rows_[l] -= take;
      if (cfg_.mode == Mode::SealedBatch && layer_rows_[l] == 0) sealed_[l] = 0;
      ++st_.firings;
      st_.fired_rows += take;
      return true;
    }
  }
  return false;
}

uint32_t ExpertQueue::slot_rows(uint32_t layer, uint32_t expert) const {
  if (layer >= cfg_.layer_count || expert >= cfg_.expert_count) fail(Status::InvalidArgument, "expert queue: index");
  return slot(layer, expert).count;
}

}  // namespace eq
}  // namespace spc
