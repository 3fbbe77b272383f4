#include "topology_switch.h"

namespace spc {
namespace ts {

uint64_t kv_key(uint64_t ns, uint64_t content_hash) {
  uint8_t b[8];
  put_u64(b, content_hash);
  return fnv1a64(b, 8, ns) | 1;  // never zero: zero marks an unhashed tier slot
}

uint64_t manifest_key(uint64_t ns, uint64_t sequence_id) {
  uint8_t b[8];
  put_u64(b, sequence_id);
  return kv_key(ns, fnv1a64(b, 8, kManifestDomain) | 1);
}

Budget estimate_budget(const Config& c, const Recipe& target, uint32_t active, uint64_t warm_kv_bytes) {
  if (!c.read_bytes_per_s || !c.write_bytes_per_s) fail(Status::InvalidArgument, "topology switch: zero bandwidth");
  Budget b;
  b.quiesce_us = c.step_time_us;
  b.checkpoint_us = uint64_t(active) * c.manifest_block_bytes * 1000000ull / c.write_bytes_per_s;
  b.swap_fixed_us = c.swap_fixed_us;
  b.swap_stream_us = target.weight_pack_bytes * 1000000ull / c.read_bytes_per_s;
  b.resume_warm_us = warm_kv_bytes * 1000000ull / c.read_bytes_per_s;  // overlapped with decode: not in total
  b.total_us = b.quiesce_us + b.checkpoint_us + b.swap_fixed_us + b.swap_stream_us;
  return b;
}

TopologySwitch::TopologySwitch(const Config& c, Tier* tier, SwapDevice* swap, ManifestWriter* writer)
    : cfg_(c), tier_(tier), swap_(swap), writer_(writer), current_(c.initial), target_(c.initial) {
  if (!tier || !swap || !writer) fail(Status::InvalidArgument, "topology switch: missing seam");
  if (!c.max_sequences || !c.max_blocks_per_sequence || !c.step_time_us)
    fail(Status::InvalidArgument, "topology switch: zero capacity or step time");
  if (!c.read_bytes_per_s || !c.write_bytes_per_s) fail(Status::InvalidArgument, "topology switch: zero bandwidth");
  if (kManifestHeaderBytes + uint64_t(c.max_blocks_per_sequence) * 8 > c.manifest_block_bytes)
    fail(Status::InvalidArgument, "topology switch: manifest record cannot hold a full block list");
  seqs_.resize(c.max_sequences);
  keys_.assign(size_t(c.max_sequences) * c.max_blocks_per_sequence, 0);
}

int TopologySwitch::find(uint64_t id) const {
  for (size_t i = 0; i < seqs_.size(); ++i)
    if (seqs_[i].slot != Slot::Free && seqs_[i].id == id) return int(i);
  return -1;
}

void TopologySwitch::track_sequence(uint64_t id, uint64_t recipe) {
  if (!id) fail(Status::InvalidArgument, "topology switch: zero sequence id");
  if (state_ != State::Steady) fail(Status::Busy, "topology switch: admissions closed during a switch");
  if (recipe != current_.recipe_id) fail(Status::InvalidArgument, "topology switch: sequence of another recipe");
  if (find(id) >= 0) fail(Status::Duplicate, "topology switch: sequence already tracked");
  for (Seq& s : seqs_) {
    if (s.slot != Slot::Free) continue;
    s = Seq{};
    s.id = id;
    s.recipe = recipe;
    s.slot = Slot::Active;
    ++tracked_;
    return;
  }
  fail(Status::CapacityExceeded, "topology switch: sequence table full");
}

void TopologySwitch::set_sequence_kv(uint64_t id, uint32_t position, const std::vector<uint64_t>& hashes) {
  if (hashes.size() > cfg_.max_blocks_per_sequence) fail(Status::CapacityExceeded, "topology switch: too many blocks");
  const int i = find(id);
  if (i < 0) fail(Status::NotFound, "topology switch: unknown sequence");
  if (seqs_[i].checkpointed) fail(Status::Busy, "topology switch: block set frozen by a checkpoint");
  uint64_t* k = keys_of(i);
  for (size_t j = 0; j < hashes.size(); ++j) k[j] = kv_key(cfg_.kv_namespace, hashes[j]);
  seqs_[i].blocks = uint32_t(hashes.size());
  seqs_[i].position = position;
}

void TopologySwitch::sequence_at_boundary(uint64_t id) {
  const int i = find(id);
  if (i < 0) fail(Status::NotFound, "topology switch: unknown sequence");
  seqs_[i].slot = Slot::AtBoundary;
}

void TopologySwitch::sequence_complete(uint64_t id) {
  const int i = find(id);
  if (i < 0) fail(Status::NotFound, "topology switch: unknown sequence");
  Seq& s = seqs_[i];
  if (s.pinned) {
    const uint64_t* k = keys_of(i);
    for (uint32_t j = 0; j < s.blocks; ++j) tier_->pin(k[j], false);
  }
  if (state_ != State::Steady && !s.checkpointed) ++st_.completed_mid_switch;
  s.slot = Slot::Free;
  s.resume = ResumeClass::Pending;
  s.blocks = 0;
  --tracked_;
}

void TopologySwitch::begin(const Recipe& target) {
  if (!target.recipe_id) fail(Status::InvalidArgument, "topology switch: zero recipe id");
  if (state_ != State::Steady) fail(Status::Busy, "topology switch: a switch is already running");
  if (target.recipe_id == current_.recipe_id)
    fail(Status::InvalidArgument, "topology switch: target is the running recipe");
  target_ = target;
  state_ = State::Quiesce;
  cursor_ = 0;
  swap_started_ = false;
  last_error_ = Status::Ok;
}

Status TopologySwitch::checkpoint(size_t i) {
  Seq& s = seqs_[i];
  const uint64_t* k = keys_of(i);
  if (!s.pinned) {
    // pin before any manifest reservation: reserving a write is the tier's
    // only eviction path, so an unpinned block could be evicted by it
    for (uint32_t j = 0; j < s.blocks; ++j) {
      const Status r = tier_->pin(k[j], true);
      if (r == Status::Ok) {
        ++st_.tier_blocks_found;
        ++st_.blocks_pinned;
      } else if (r == Status::NotFound) {
        ++st_.tier_blocks_absent;  // never written back: resume will recompute
      } else {
        return r;
      }
    }
    s.pinned = true;
  }
  std::string rec(cfg_.manifest_block_bytes, '\0');
  uint8_t* p = reinterpret_cast<uint8_t*>(&rec[0]);
  put_u64(p, s.id);
  put_u64(p + 8, s.recipe);
  put_u32(p + 16, s.position);
  put_u32(p + 20, s.blocks);
  for (uint32_t j = 0; j < s.blocks; ++j) put_u64(p + kManifestHeaderBytes + 8 * j, k[j]);
  WriteReservation res;
  Status r = tier_->reserve_write(manifest_key(cfg_.kv_namespace, s.id), &res);
  if (r != Status::Ok) return r;
  if (!res.already_present) {
    r = writer_->write_block(res.device_offset, rec);
    if (r != Status::Ok) {
      tier_->abort_write(res);
      return r;
    }
    r = tier_->commit_write(res);
    if (r != Status::Ok) return r;
  }
  s.checkpointed = true;
  ++st_.sequences_checkpointed;
  ++st_.manifest_writes;
  st_.manifest_bytes += cfg_.manifest_block_bytes;
  return Status::Ok;
}

bool TopologySwitch::checkpoint_all() {
  for (; cursor_ < seqs_.size(); ++cursor_) {
    if (seqs_[cursor_].slot == Slot::Free || seqs_[cursor_].checkpointed) continue;
    const Status r = checkpoint(cursor_);
    if (r != Status::Ok) {
      last_error_ = r;  // retried from this sequence on the next advance
      return false;
    }
  }
  return true;
}

void TopologySwitch::resume(size_t i, uint32_t step_now) {
  Seq& s = seqs_[i];
  const uint64_t* k = keys_of(i);
  bool warm = true;
  for (uint32_t j = 0; j < s.blocks; ++j) {
    uint64_t off;
    if (tier_->offset_of(k[j], &off) != Status::Ok) warm = false;
    tier_->pin(k[j], false);
  }
  if (warm && s.blocks) {
    std::vector<TierNeed> needs;
    for (uint32_t j = 0; j < s.blocks; j += kPlanChunk) {
      needs.clear();
      for (uint32_t q = j; q < s.blocks && q < j + kPlanChunk; ++q) needs.push_back(TierNeed{k[q], step_now + 1});
      tier_->plan_lookahead(needs, step_now);  // a failed plan costs prefetch only
    }
    s.resume = ResumeClass::Warm;
    ++st_.resumed_warm;
  } else {
    s.resume = ResumeClass::Recompute;
    ++st_.resumed_recompute;
  }
}

State TopologySwitch::advance(uint32_t step_now) {
  if (state_ == State::Quiesce) {
    bool drained = true;
    for (const Seq& s : seqs_)
      if (s.slot == Slot::Active) drained = false;
    if (drained) {
      state_ = State::Checkpoint;
      cursor_ = 0;
    }
  }
  if (state_ == State::Checkpoint && checkpoint_all()) {
    state_ = State::Swap;
    swap_started_ = false;
  }
  if (state_ == State::Swap) {
    bool issued = true;
    if (!swap_started_) {
      const Status r = swap_->begin_swap(current_, target_);
      if (r == Status::Ok) {
        swap_started_ = true;
        ++st_.swaps_started;
      } else {
        last_error_ = r;
        issued = false;
      }
    }
    if (issued) {
      const Status r = swap_->poll_swap();
      if (r == Status::Ok) {
        state_ = State::Resume;
        cursor_ = 0;
      } else if (r != Status::Busy) {
        last_error_ = r;
      }
    }
  }
  if (state_ == State::Resume) {
    for (; cursor_ < seqs_.size(); ++cursor_)
      if (seqs_[cursor_].slot != Slot::Free) resume(cursor_, step_now);
    current_ = target_;
    state_ = State::Steady;
    last_error_ = Status::Ok;
    ++st_.switches_completed;
  }
  return state_;
}

ResumeClass TopologySwitch::resume_class_of(uint64_t id) const {
  const int i = find(id);
  return i < 0 ? ResumeClass::Recompute : seqs_[i].resume;
}

}  // namespace ts
}  // namespace spc
