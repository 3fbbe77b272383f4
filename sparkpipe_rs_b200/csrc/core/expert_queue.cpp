#include "expert_queue.h"

#include <algorithm>

namespace spc {
namespace eq {

void ExpertQueue::Ring::push(const Row& r) {
  if (n_ == buf_.size()) {  // full: unroll into a buffer twice the size
    std::vector<Row> grown(std::max<size_t>(8, buf_.size() * 2));
    for (uint32_t i = 0; i < n_; ++i) grown[i] = buf_[(head_ + i) & (buf_.size() - 1)];
    buf_.swap(grown);
    head_ = 0;
  }
  buf_[(head_ + n_) & (buf_.size() - 1)] = r;
  ++n_;
}

ExpertQueue::Row ExpertQueue::Ring::pop() {
  const Row r = buf_[head_];
  head_ = (head_ + 1) & uint32_t(buf_.size() - 1);
  --n_;
  return r;
}

ExpertQueue::ExpertQueue(const Config& c) : cfg_(c) {
  if (c.layer_count == 0 || c.layer_count > kMaxLayers) fail(Status::InvalidArgument, "expert queue: layer count");
  if (c.expert_count == 0 || c.expert_count > kMaxExperts) fail(Status::InvalidArgument, "expert queue: expert count");
  if (c.firing_threshold_rows == 0 || c.firing_threshold_rows > kMaxFiringRows)
    fail(Status::InvalidArgument, "expert queue: firing threshold must be 1..1024 rows");
  if (c.firing_deadline_ns == 0) fail(Status::InvalidArgument, "expert queue: firing deadline must be positive");
  if (c.mode != Mode::LowLatency && c.mode != Mode::SealedBatch) fail(Status::InvalidArgument, "expert queue: mode");
  const uint32_t slots = c.layer_count * c.expert_count;
  rings_.resize(slots);
  layers_.resize(c.layer_count);
  while (leaves_ < slots) leaves_ <<= 1;
  tree_.assign(2 * size_t(leaves_), kNever);
}

uint64_t ExpertQueue::due_key(uint32_t slot) const {
  const Ring& r = rings_[slot];
  if (r.size() == 0) return kNever;
  if (cfg_.mode == Mode::SealedBatch) return layers_[slot / cfg_.expert_count].sealed ? 0 : kNever;
  if (r.size() >= cfg_.firing_threshold_rows) return 0;
  const uint64_t oldest = r.front().arrival_ns;
  // due once now - oldest >= deadline; a sum past 2^64 - 1 is never reached by a clock
  return oldest > kNever - cfg_.firing_deadline_ns ? kNever : oldest + cfg_.firing_deadline_ns;
}

void ExpertQueue::refresh(uint32_t slot) {
  uint32_t i = leaves_ + slot;
  tree_[i] = due_key(slot);
  for (i >>= 1; i; i >>= 1) tree_[i] = std::min(tree_[2 * i], tree_[2 * i + 1]);
}

void ExpertQueue::refresh_layer(uint32_t layer) {
  for (uint32_t e = 0; e < cfg_.expert_count; ++e) refresh(index(layer, e));
}

int ExpertQueue::leftmost_due(uint64_t now_ns) const {
  // A key of kNever marks an empty (or never-due) slot even when now_ns is kNever.
  const uint64_t limit = std::min(now_ns, kNever - 1);
  if (tree_[1] > limit) return -1;
  uint32_t i = 1;
  while (i < leaves_) i = tree_[2 * i] <= limit ? 2 * i : 2 * i + 1;
  return int(i - leaves_);
}

void ExpertQueue::enqueue(uint32_t layer, uint32_t expert, uint64_t row_id, uint64_t arrival_ns) {
  if (layer >= cfg_.layer_count || expert >= cfg_.expert_count) fail(Status::InvalidArgument, "expert queue: index");
  Layer& L = layers_[layer];
  if (cfg_.mode == Mode::SealedBatch && L.sealed) fail(Status::Busy, "expert queue: layer is sealed");
  if (queued_ >= kMaxRows) fail(Status::CapacityExceeded, "expert queue: row capacity exhausted");
  const uint32_t s = index(layer, expert);
  Ring& r = rings_[s];
  r.push(Row{row_id, arrival_ns});
  ++queued_;
  ++L.rows;
  st_.enqueued = queued_;
  // the key moves only when the slot gets its first row or reaches the threshold
  if (r.size() == 1 || r.size() == cfg_.firing_threshold_rows) refresh(s);
}

void ExpertQueue::seal(uint32_t layer) {
  if (layer >= cfg_.layer_count) fail(Status::InvalidArgument, "expert queue: layer");
  if (cfg_.mode != Mode::SealedBatch) fail(Status::Unsupported, "expert queue: sealing needs the sealed-batch mode");
  Layer& L = layers_[layer];
  if (L.sealed) fail(Status::Busy, "expert queue: layer already sealed");
  if (L.rows == 0) fail(Status::NotFound, "expert queue: nothing to seal");
  for (uint32_t e = 0; e < cfg_.expert_count; ++e)
    if (rings_[index(layer, e)].size() > kMaxFiringRows)
      fail(Status::CapacityExceeded, "expert queue: a slot holds more rows than one firing");
  L.sealed = true;
  refresh_layer(layer);
}

void ExpertQueue::set_firing_threshold(uint32_t rows) {
  if (rows == 0 || rows > kMaxFiringRows) fail(Status::InvalidArgument, "expert queue: firing threshold");
  cfg_.firing_threshold_rows = rows;
  for (uint32_t s = 0; s < rings_.size(); ++s) refresh(s);
}

bool ExpertQueue::next_firing(uint64_t now_ns, Firing& out) {
  const int found = leftmost_due(now_ns);
  if (found < 0) return false;
  const uint32_t s = uint32_t(found);
  Ring& r = rings_[s];
  Layer& L = layers_[s / cfg_.expert_count];
  const uint32_t take = cfg_.mode == Mode::SealedBatch ? r.size() : std::min(r.size(), kMaxFiringRows);
  out.layer = s / cfg_.expert_count;
  out.expert = s % cfg_.expert_count;
  out.row_ids.resize(take);
  for (uint32_t i = 0; i < take; ++i) out.row_ids[i] = r.pop().id;
  queued_ -= take;
  L.rows -= take;
  st_.enqueued = queued_;
  ++st_.firings;
  st_.fired_rows += take;
  if (cfg_.mode == Mode::SealedBatch && L.rows == 0) {
    L.sealed = false;  // drained: the layer takes rows again
    refresh_layer(out.layer);
  } else {
    refresh(s);
  }
  return true;
}

uint32_t ExpertQueue::slot_rows(uint32_t layer, uint32_t expert) const {
  if (layer >= cfg_.layer_count || expert >= cfg_.expert_count) fail(Status::InvalidArgument, "expert queue: index");
  return rings_[index(layer, expert)].size();
}

}  // namespace eq
}  // namespace spc
