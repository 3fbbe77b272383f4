#include "memory.h"

#include <algorithm>
#include <queue>
#include <tuple>

namespace spc {

// ============================================================== KvArena
KvArena::KvArena(const KvArenaConfig& c) {
  if (c.physical_block_count == 0 || c.block_token_count == 0 || c.block_token_count > kKvMaxBlockTokens ||
      c.resident_block_capacity > c.physical_block_count || c.layer_count == 0 || c.layer_count > kKvMaxLayers ||
      c.kv_head_count == 0 || c.head_dim == 0 || c.bytes_per_scalar == 0 || c.key_device_base == 0 ||
      (c.value_device_base == 0 && c.value_block_stride_bytes != 0))
    fail(Status::InvalidArgument, "KvArena: invalid configuration");
  n_ = c.physical_block_count;
  block_tokens_ = c.block_token_count;
  resident_cap_ = c.resident_block_capacity ? c.resident_block_capacity : c.physical_block_count;
  layers_ = c.layer_count;
  heads_ = c.kv_head_count;
  dim_ = c.head_dim;
  bytes_ = c.bytes_per_scalar;
  const uint64_t def = uint64_t(block_tokens_) * layers_ * heads_ * dim_ * bytes_;
  const bool has_value = c.value_device_base != 0 || c.value_block_stride_bytes != 0;
  key_stride_ = c.key_block_stride_bytes ? c.key_block_stride_bytes : def;
  value_stride_ = has_value ? (c.value_block_stride_bytes ? c.value_block_stride_bytes : def) : 0;
  key_base_ = c.key_device_base;
  value_base_ = has_value ? c.value_device_base : 0;
  reset();
}

KvArena::Block KvArena::fresh(uint32_t b) const {
  Block k;
  k.key_addr = key_base_ + key_stride_ * b;
  k.value_addr = value_base_ ? value_base_ + value_stride_ * b : 0;
  return k;
}

void KvArena::reset() {
  blocks_.assign(n_, Block());
  for (uint32_t b = 0; b < n_; ++b) blocks_[b] = fresh(b);
  free_bits_.assign((n_ + 63) / 64, ~0ull);
  if (n_ % 64) free_bits_.back() = (1ull << (n_ % 64)) - 1;
  free_count_ = n_;
  // cumulative eviction / stall counters survive a reset, the others do not
  epoch_ = allocated_ = recycled_ = resident_ = retained_ = released_ = 0;
}

void KvArena::set_free_bit(uint32_t b, bool free) {
  uint64_t& w = free_bits_[b >> 6];
  const uint64_t m = 1ull << (b & 63);
  const bool was = (w & m) != 0;
  if (free && !was) { w |= m; ++free_count_; }
  if (!free && was) { w &= ~m; --free_count_; }
}

KvArena::Block& KvArena::checked(uint32_t b) {
  if (b >= n_) fail(Status::InvalidArgument, "KvArena: block index out of range");
  return blocks_[b];
}

uint32_t KvArena::acquire_block() {
  for (size_t w = 0; w < free_bits_.size(); ++w) {
    if (free_bits_[w]) {
      const uint32_t b = uint32_t(w * 64 + __builtin_ctzll(free_bits_[w]));
      Block& k = blocks_[b];
      ++epoch_;
      k.flags = kBlockAllocated;
      k.refs = 0;
      ++k.generation;
      k.epoch = epoch_;
      set_free_bit(b, false);
      ++allocated_;
      return b;
    }
  }
  fail(Status::CapacityExceeded, "KvArena: no free block");
}

void KvArena::recycle_block(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated)) fail(Status::InvalidArgument, "KvArena: recycle of a free block");
  if (k.refs) fail(Status::Busy, "KvArena: recycle of a referenced block");
  ++epoch_;
  if ((k.flags & kBlockResident) && resident_) --resident_;
  k.flags = kBlockAllocated;
  ++k.generation;
  k.epoch = epoch_;
  ++recycled_;
}

void KvArena::retain_block(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated)) fail(Status::InvalidArgument, "KvArena: retain of a free block");
  ++epoch_;
  ++k.refs;
  k.epoch = epoch_;
  ++retained_;
}

void KvArena::release_block_reference(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated) || k.refs == 0) fail(Status::InvalidArgument, "KvArena: release below zero");
  ++epoch_;
  --k.refs;
  k.epoch = epoch_;
  ++released_;
}

uint32_t KvArena::pick_victim(const std::vector<uint32_t>& prot) const {
  uint32_t best = kNoBlock;
  for (uint32_t b = 0; b < n_; ++b) {
    const Block& k = blocks_[b];
    if (!(k.flags & kBlockAllocated) || !(k.flags & kBlockResident)) continue;
    if (std::find(prot.begin(), prot.end(), b) != prot.end()) continue;
    if (best == kNoBlock || std::make_pair(k.refs, k.epoch) < std::make_pair(blocks_[best].refs, blocks_[best].epoch))
      best = b;
  }
  return best;
}

uint32_t KvArena::trim_inner(const std::vector<uint32_t>& prot, uint32_t target) {
  uint32_t ev = 0;
  while (resident_ > target) {
    const uint32_t v = pick_victim(prot);
    if (v == kNoBlock) {
      ++stalls_;
      fail(Status::CapacityExceeded, "KvArena: no resident block can be evicted");
    }
    ++epoch_;
    Block& k = blocks_[v];
    k.flags &= ~kBlockResident;
    if (resident_) --resident_;
    k.epoch = epoch_;
    ++evicted_;
    ++ev;
  }
  return ev;
}

void KvArena::make_room(uint32_t b) {
  if (resident_ + 1 <= resident_cap_) return;
  trim_inner({b}, resident_cap_ - 1);
}

void KvArena::mark_block_resident(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated)) fail(Status::InvalidArgument, "KvArena: resident mark of a free block");
  if (!(k.flags & kBlockResident)) {
    make_room(b);
    ++resident_;
  }
  ++epoch_;
  blocks_[b].flags |= kBlockResident;
  blocks_[b].epoch = epoch_;
}

void KvArena::mark_block_nonresident(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated)) fail(Status::InvalidArgument, "KvArena: nonresident mark of a free block");
  ++epoch_;
  if (k.flags & kBlockResident) {
    k.flags &= ~kBlockResident;
    if (resident_) --resident_;
  }
  k.epoch = epoch_;
}

void KvArena::free_block(uint32_t b) {
  Block& k = checked(b);
  if (!(k.flags & kBlockAllocated)) return;  // freeing a free block is a no-op
  if (k.refs) fail(Status::Busy, "KvArena: free of a referenced block");
  ++epoch_;
  if ((k.flags & kBlockResident) && resident_) --resident_;
  k.flags = 0;
  ++k.generation;
  k.epoch = epoch_;
  set_free_bit(b, true);
}

KvBlockView KvArena::resolve_block(uint32_t b) const {
  if (b >= n_) fail(Status::InvalidArgument, "KvArena: block index out of range");
  const Block& k = blocks_[b];
  if (!(k.flags & kBlockAllocated)) fail(Status::NotFound, "KvArena: block not allocated");
  return KvBlockView{b, block_tokens_, layers_, heads_, dim_, bytes_, k.generation, key_stride_, value_stride_,
                     k.key_addr, k.value_addr};
}

uint32_t KvArena::trim_resident_blocks(const std::vector<uint32_t>& prot, uint32_t target) {
  if (target > resident_cap_) fail(Status::InvalidArgument, "KvArena: trim target above capacity");
  return trim_inner(prot, target);
}

uint32_t KvArena::evict_resident_blocks_to_limit(uint32_t max_resident, const std::vector<uint32_t>& prot) {
  uint32_t ev = 0;
  while (resident_ > max_resident) {
    const uint32_t v = pick_victim(prot);
    if (v == kNoBlock) break;
    mark_block_nonresident(v);
    ++evicted_;
    ++ev;
  }
  return ev;
}

// ============================================================== Arena
static constexpr uint32_t kNoSlot = 0xffffffffu;
static constexpr uint32_t kInUse = 0xfffffffeu;

Arena::Arena(const std::vector<ArenaClass>& cls) {
  if (cls.empty() || cls.size() > kMaxClasses) fail(Status::InvalidArgument, "Arena: 1..8 size classes");
  uint64_t prev = 0, total = 0;
  for (const auto& c : cls) {
    const uint64_t sb = (uint64_t(c.slot_bytes) + kAlignment - 1) & ~uint64_t(kAlignment - 1);
    if (c.slot_bytes == 0 || c.slot_count == 0) fail(Status::InvalidArgument, "Arena: empty size class");
    if (total > 0 && sb <= prev) fail(Status::InvalidArgument, "Arena: slot sizes must strictly increase");
    total += sb * c.slot_count;
    prev = sb;
  }
  backing_.assign(total, 0);
  size_t off = 0;
  for (const auto& c : cls) {
    Cls k;
    k.slot_bytes = uint32_t((uint64_t(c.slot_bytes) + kAlignment - 1) & ~uint64_t(kAlignment - 1));
    k.slot_count = c.slot_count;
    k.offset = off;
    off += size_t(k.slot_bytes) * k.slot_count;
    k.next.resize(c.slot_count);
    for (uint32_t i = 0; i < c.slot_count; ++i) k.next[i] = i + 1 < c.slot_count ? i + 1 : kNoSlot;
    k.gen.assign(c.slot_count, 0);
    k.head = 0;
    k.free_count = c.slot_count;
    k.generation = 0;
    classes_.push_back(std::move(k));
  }
}

ArenaHandle Arena::acquire(uint32_t bytes) {
  if (bytes == 0) fail(Status::InvalidArgument, "Arena: zero-byte request");
  for (uint32_t ci = 0; ci < classes_.size(); ++ci) {
    Cls& c = classes_[ci];
    if (bytes > c.slot_bytes) continue;
    if (c.free_count == 0) fail(Status::CapacityExceeded, "Arena: size class exhausted");
    const uint32_t s = c.head;
    c.head = c.next[s];
    c.next[s] = kInUse;
    --c.free_count;
    ++c.generation;
    ++c.gen[s];
    return ArenaHandle{ci, s, c.gen[s]};
  }
  fail(Status::CapacityExceeded, "Arena: request larger than every size class");
}

bool Arena::live(const ArenaHandle& h) const {
  if (h.class_index >= classes_.size()) return false;
  const Cls& c = classes_[h.class_index];
  return h.slot_index < c.slot_count && c.next[h.slot_index] == kInUse && c.gen[h.slot_index] == h.generation;
}

void Arena::release(const ArenaHandle& h) {
  if (!live(h)) fail(Status::NotFound, "Arena: stale or foreign handle");
  Cls& c = classes_[h.class_index];
  c.next[h.slot_index] = c.head;
  c.head = h.slot_index;
  ++c.free_count;
  ++c.generation;
}

uint8_t* Arena::get(const ArenaHandle& h) {
  if (!live(h)) return nullptr;
  const Cls& c = classes_[h.class_index];
  return backing_.data() + c.offset + size_t(h.slot_index) * c.slot_bytes;
}

// ============================================================== StatePool
StatePool::StatePool(uint32_t slot_count, uint64_t slot_bytes) : slot_bytes_(slot_bytes) {
  if (slot_count == 0 || slot_bytes == 0) fail(Status::InvalidArgument, "StatePool: empty pool");
  backing_.assign(size_t(slot_bytes) * slot_count, 0);
  next_.resize(slot_count);
  for (uint32_t i = 0; i < slot_count; ++i) next_[i] = i + 1 < slot_count ? i + 1 : kNoSlot;
  head_ = 0;
  free_count_ = slot_count;
}

int64_t StatePool::acquire() {
  if (free_count_ == 0) return -1;
  const uint32_t s = head_;
  head_ = next_[s];
  next_[s] = kInUse;
  --free_count_;
  return s;
}

void StatePool::release(uint32_t s) {
  if (s >= next_.size() || next_[s] != kInUse) fail(Status::NotFound, "StatePool: slot not in use");
  next_[s] = head_;
  head_ = s;
  ++free_count_;
}

bool StatePool::in_use(uint32_t s) const { return s < next_.size() && next_[s] == kInUse; }

uint8_t* StatePool::slot(uint32_t s) {
  if (!in_use(s)) return nullptr;
  return backing_.data() + size_t(s) * slot_bytes_;
}

// ============================================================== BatchSequenceTable
BatchSequenceTable::BatchSequenceTable(uint32_t capacity, uint32_t lane_count) : cap_(capacity), lanes_(lane_count) {
  if (capacity == 0 || capacity > kMaxSequences || lane_count == 0)
    fail(Status::InvalidArgument, "BatchSequenceTable: invalid capacity / lanes");
  seqs_.resize(capacity);
}

uint32_t BatchSequenceTable::resolve(uint32_t handle) const {
  const uint32_t idx = handle & ((1u << kIndexBits) - 1);
  if (idx >= cap_ || seqs_[idx].generation != (handle >> kIndexBits))
    fail(Status::NotFound, "BatchSequenceTable: stale handle");
  return idx;
}

uint32_t BatchSequenceTable::admit(uint64_t id, uint32_t ctx, uint32_t frag_base, uint32_t frag_count) {
  if (frag_count == 0) fail(Status::InvalidArgument, "BatchSequenceTable: zero fragments");
  uint32_t idx;
  if (free_head_ != 0xffffffffu) {
    idx = free_head_;
    free_head_ = seqs_[idx].free_next;
  } else if (high_water_ < cap_) {
    idx = high_water_++;
  } else {
    fail(Status::CapacityExceeded, "BatchSequenceTable: full");
  }
  BatchSequence& s = seqs_[idx];
  s.sequence_id = id;
  s.state = SeqState::Active;
  s.lane_count = lanes_;
  s.exchange_number = 0;
  s.context_tokens = ctx;
  s.fragment_base = frag_base;
  s.fragment_count = frag_count;
  ++active_;
  ++exchanges_;
  return idx | (s.generation << kIndexBits);
}

void BatchSequenceTable::begin_exchange(uint32_t h, uint32_t appended) {
  BatchSequence& s = seqs_[resolve(h)];
  if (s.state != SeqState::AwaitingTool) fail(Status::InvalidArgument, "begin_exchange: not awaiting a tool");
  s.state = SeqState::Active;
  ++s.exchange_number;
  s.context_tokens += appended;
  --awaiting_;
  ++active_;
  ++exchanges_;
}

void BatchSequenceTable::pause_for_tool(uint32_t h) {
  BatchSequence& s = seqs_[resolve(h)];
  if (s.state != SeqState::Active) fail(Status::InvalidArgument, "pause_for_tool: not active");
  s.state = SeqState::AwaitingTool;
  --active_;
  ++awaiting_;
}

void BatchSequenceTable::complete(uint32_t h) {
  const uint32_t idx = resolve(h);
  BatchSequence& s = seqs_[idx];
  if (s.state != SeqState::Active && s.state != SeqState::AwaitingTool)
    fail(Status::InvalidArgument, "complete: sequence not live");
  if (s.state == SeqState::Active) --active_;
  else --awaiting_;
  s.state = SeqState::Complete;
  ++s.generation;
  s.free_next = free_head_;
  free_head_ = idx;
  ++complete_;
}

const BatchSequence& BatchSequenceTable::sequence(uint32_t h) const { return seqs_[resolve(h)]; }

uint32_t BatchSequenceTable::firing_threshold(uint32_t topk, uint32_t experts, uint32_t cap) const {
  if (experts == 0 || cap == 0) return 1;
  uint32_t t = (active_ * lanes_ * topk) / experts;
  if (t == 0) t = 1;
  return std::min(t, cap);
}

// ============================================================== row allocator
static uint32_t alpha_milli(uint32_t ema) {
  if (ema <= 1000) return 0;
  const uint32_t a = uint32_t((uint64_t(ema - 1000) * 1000) / ema);
  return std::min<uint32_t>(a, 999);
}

uint32_t row_allocator_assign(const std::vector<RowSlot>& slots, uint32_t cap, uint32_t cost_milli,
                              std::vector<uint32_t>& budgets) {
  budgets.assign(slots.size(), 0);
  if (cap == 0) return 0;
  const uint32_t n = (uint32_t)slots.size();
  const uint32_t base = std::min(n, cap);
  uint32_t remaining = cap - base;
  // probes: fixed two-row grants in slot order, capacity permitting
  for (uint32_t i = 0; i < n && remaining; ++i) {
    if (!slots[i].probe || !slots[i].maximum_draft_depth) continue;
    const uint32_t g = std::min({2u, slots[i].maximum_draft_depth, remaining});
    budgets[i] = g;
    remaining -= g;
  }
  // value-ranked grants: each slot's marginal value decays geometrically, so a
  // max-heap of next values (ties -> lower index) reproduces the greedy order.
  const uint32_t cost = cost_milli ? cost_milli : 1000;
  using Item = std::tuple<uint32_t, int64_t>;  // (value, -index)
  std::priority_queue<Item> heap;
  std::vector<uint32_t> next_value(n, 0);
  for (uint32_t i = 0; i < n; ++i) {
    if (slots[i].probe || slots[i].maximum_draft_depth == 0) continue;
    const uint32_t a = alpha_milli(slots[i].commit_ema_milli);
    if (!a) continue;
    next_value[i] = uint32_t(uint64_t(a) * 1000 / cost);
    if (next_value[i]) heap.emplace(next_value[i], -int64_t(i));
  }
  while (remaining && !heap.empty()) {
    auto [v, ni] = heap.top();
    heap.pop();
    const uint32_t i = uint32_t(-ni);
    ++budgets[i];
    --remaining;
    if (budgets[i] < slots[i].maximum_draft_depth) {
      const uint32_t a = alpha_milli(slots[i].commit_ema_milli);
      const uint32_t nv = uint32_t(uint64_t(v) * a / 1000);
      if (nv) heap.emplace(nv, ni);
    }
  }
  uint32_t total = base;
  for (uint32_t b : budgets) total += b;
  return total;
}

}  // namespace spc
