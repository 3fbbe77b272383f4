#include "prefix_cache.h"

#include <algorithm>

namespace spc {

namespace {
constexpr uint64_t kContentSeed = 7809847782465536322ull;
constexpr uint32_t kGoldenGamma32 = 0x9e3779b9u;

inline uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v;
  h *= kFnv64Prime;
  h ^= h >> 32;
  return h;
}
}  // namespace

uint64_t prefix_hash_block(const uint32_t* t, uint32_t n, uint64_t parent) {
  uint64_t h = parent ^ kFnv64Prime;
  for (uint32_t i = 0; i < n; ++i) h = mix(h, uint64_t(t[i]) + (uint64_t(i) << 32));
  return mix(h, n);
}

uint64_t prefix_content_hash(const uint32_t* t, uint32_t n) {
  uint64_t h = kContentSeed;
  for (uint32_t i = 0; i < n; ++i) h = mix(h, (uint64_t(t[i]) << 1) ^ uint64_t(uint32_t(i + kGoldenGamma32)));
  return mix(h, n);
}

PromptHash prefix_hash_prompt(uint32_t bt, uint64_t parent, const uint32_t* t, uint32_t n) {
  if (bt == 0 || bt > kPrefixMaxBlockTokens) fail(Status::InvalidArgument, "prefix hash: block size 1..256");
  PromptHash r;
  r.token_count = r.hashed_token_count = n;
  r.parent_hash = parent;
  uint64_t h = parent;
  for (uint32_t off = 0; off < n; off += bt) {
    const uint32_t len = std::min(bt, n - off);
    h = prefix_hash_block(t + off, len, h);
    ++r.block_count;
  }
  r.last_block_token_count = n ? (n - 1) % bt + 1 : 0;
  r.prompt_hash = h;
  return r;
}

static KvArenaConfig arena_cfg(uint32_t bt, uint32_t blocks) {
  KvArenaConfig c;
  c.physical_block_count = blocks;
  c.block_token_count = bt;
  c.key_device_base = 1;  // block addresses are resolved by the device cache tensor, not here
  return c;
}

PrefixCache::PrefixCache(uint32_t bt, uint32_t blocks, uint32_t max_sequences)
    : block_tokens_(bt), max_sequences_(max_sequences), arena_(arena_cfg(bt, blocks)) {
  if (bt == 0 || bt > kPrefixMaxBlockTokens) fail(Status::InvalidArgument, "PrefixCache: block size 1..256");
  if (max_sequences == 0) fail(Status::InvalidArgument, "PrefixCache: zero sequences");
  reset();
}

void PrefixCache::reset() {
  arena_.reset();
  entries_.clear();
  for (const auto& kv : host_entries_) host_free_.push_back(kv.second.slot);
  host_entries_.clear();
  host_lru_.clear();
  host_free_.insert(host_free_.end(), host_deferred_.begin(), host_deferred_.end());
  host_deferred_.clear();
  tier_out_.clear();
  tier_in_.clear();
  seqs_.clear();
  lru_.clear();
  const uint32_t n = arena_.physical_block_count();
  block_hash_.assign(n, 0);
  block_has_entry_.assign(n, 0);
  lru_pos_.assign(n, lru_.end());
  in_lru_.assign(n, 0);
}

PrefixCache::Seq& PrefixCache::seq(uint64_t id) {
  auto it = seqs_.find(id);
  if (it == seqs_.end()) fail(Status::NotFound, "PrefixCache: unknown sequence");
  return it->second;
}
const PrefixCache::Seq& PrefixCache::seq(uint64_t id) const {
  auto it = seqs_.find(id);
  if (it == seqs_.end()) fail(Status::NotFound, "PrefixCache: unknown sequence");
  return it->second;
}

void PrefixCache::retain(uint32_t b) {
  if (in_lru_[b]) {
    lru_.erase(lru_pos_[b]);
    in_lru_[b] = 0;
  }
  arena_.retain_block(b);
}

void PrefixCache::drop(uint32_t b) {
  arena_.release_block_reference(b);
  if (arena_.reference_count(b) != 0) return;
  if (block_has_entry_[b]) {
    lru_.push_back(b);  // warm: kept until room is needed
    lru_pos_[b] = std::prev(lru_.end());
    in_lru_[b] = 1;
  } else {
    arena_.free_block(b);
  }
}

uint32_t PrefixCache::evict_one() {
  // the oldest unprotected warm block, else the protected one with the least demand
  auto victim = lru_.end();
  const Entry* best = nullptr;
  for (auto it = lru_.begin(); it != lru_.end(); ++it) {
    const Entry& e = entries_.at(block_hash_[*it]);
    if (e.protect_epoch != protect_epoch_) {
      victim = it;
      best = nullptr;
      break;
    }
    if (!best || e.protect_weight < best->protect_weight ||
        (e.protect_weight == best->protect_weight && e.protect_count < best->protect_count)) {
      best = &e;
      victim = it;
    }
  }
  if (best) ++stats_.protected_evictions;
  const uint32_t b = *victim;
  lru_.erase(victim);
  in_lru_[b] = 0;
  const uint32_t slot = host_enabled_ ? host_slot() : kNoSlot;
  if (slot != kNoSlot) {  // demote: the block's content moves to a host slot, its entry stays findable
    const uint64_t h = block_hash_[b];
    tier_out_.push_back(int32_t(b));
    tier_out_.push_back(int32_t(slot));
    host_lru_.push_back(h);
    host_entries_[h] = HostEntry{slot, entries_.at(h).content, std::prev(host_lru_.end())};
    ++stats_.demoted_blocks;
  }
  entries_.erase(block_hash_[b]);
  block_has_entry_[b] = 0;
  block_hash_[b] = 0;
  arena_.free_block(b);
  ++stats_.evicted_blocks;
  return b;
}

uint32_t PrefixCache::evict_to_free(uint32_t want) {
  uint32_t ev = 0;
  while (arena_.free_block_count() < want && !lru_.empty()) {
    evict_one();
    ++ev;
  }
  return ev;
}

void PrefixCache::reset_lookahead_protection() { ++protect_epoch_; }

void PrefixCache::enable_host_tier(uint32_t first_slot, uint32_t slots) {
  if (!slots) fail(Status::InvalidArgument, "PrefixCache: host tier without slots");
  host_enabled_ = true;
  host_free_.clear();
  for (uint32_t i = slots; i > 0; --i) host_free_.push_back(first_slot + i - 1);
}

uint32_t PrefixCache::host_slot() {
  if (host_free_.empty()) {
    // drop the oldest host entry that no reservation is promoting right now
    auto it = host_lru_.begin();
    while (it != host_lru_.end() && promoting_.count(*it)) ++it;
    if (it == host_lru_.end()) return kNoSlot;
    auto e = host_entries_.find(*it);
    host_free_.push_back(e->second.slot);
    host_entries_.erase(e);
    host_lru_.erase(it);
    ++stats_.host_dropped_blocks;
  }
  const uint32_t s = host_free_.back();
  host_free_.pop_back();
  return s;
}

void PrefixCache::take_tier_copies(std::vector<int32_t>& out, std::vector<int32_t>& in) {
  out.insert(out.end(), tier_out_.begin(), tier_out_.end());
  in.insert(in.end(), tier_in_.begin(), tier_in_.end());
  tier_out_.clear();
  tier_in_.clear();
}

void PrefixCache::release_deferred_slots() {
  host_free_.insert(host_free_.end(), host_deferred_.begin(), host_deferred_.end());
  host_deferred_.clear();
}

uint32_t PrefixCache::protect_prompt_lookahead(const uint32_t* t, uint32_t n, uint32_t weight) {
  if (n == 0) fail(Status::InvalidArgument, "PrefixCache: empty prompt");
  const uint32_t max_blocks = (n - 1) / block_tokens_;
  uint64_t h = kEmptyParentHash;
  uint32_t marked = 0;
  for (uint32_t b = 0; b < max_blocks; ++b) {
    const uint32_t* bt = t + size_t(b) * block_tokens_;
    const uint64_t nh = prefix_hash_block(bt, block_tokens_, h);
    auto it = entries_.find(nh);
    if (it == entries_.end() || it->second.content != prefix_content_hash(bt, block_tokens_)) break;
    Entry& e = it->second;
    if (e.protect_epoch != protect_epoch_) {
      e.protect_epoch = protect_epoch_;
      e.protect_weight = weight;
      e.protect_count = 1;
      ++stats_.lookahead_protections;
    } else {
      e.protect_weight = std::max(e.protect_weight, weight);
      ++e.protect_count;
    }
    h = nh;
    ++marked;
  }
  return marked;
}

uint32_t PrefixCache::cached_prefix_blocks(const std::vector<uint64_t>& chain) const {
  uint32_t n = 0;
  while (n < chain.size() && entries_.count(chain[n])) ++n;
  return n;
}

uint32_t PrefixCache::protected_warm_blocks() const {
  uint32_t n = 0;
  for (uint32_t b : lru_)
    if (entries_.at(block_hash_[b]).protect_epoch == protect_epoch_) ++n;
  return n;
}

uint32_t PrefixCache::trim_warm_blocks(uint32_t max_warm) {
  uint32_t ev = 0;
  while (lru_.size() > max_warm) {
    evict_one();
    ++ev;
  }
  stats_.trimmed_blocks += ev;
  return ev;
}

bool PrefixCache::can_allocate(uint32_t extra) const {
  return arena_.free_block_count() + lru_.size() >= extra;
}

uint32_t PrefixCache::take_block() {
  if (arena_.free_block_count() == 0) evict_to_free(1);
  const uint32_t b = arena_.acquire_block();  // throws CapacityExceeded when nothing is left
  arena_.retain_block(b);
  return b;
}

PrefixLookup PrefixCache::probe_prompt(const uint32_t* t, uint32_t n) const {
  PrefixLookup r;
  r.requested_token_count = n;
  if (n == 0) return r;
  const uint32_t max_blocks = (n - 1) / block_tokens_;
  uint64_t h = kEmptyParentHash;
  for (uint32_t b = 0; b < max_blocks; ++b) {
    const uint32_t* bt = t + size_t(b) * block_tokens_;
    const uint64_t nh = prefix_hash_block(bt, block_tokens_, h);
    auto it = entries_.find(nh);
    if (it == entries_.end() || it->second.content != prefix_content_hash(bt, block_tokens_)) {
      auto ht = host_entries_.find(nh);
      if (ht == host_entries_.end() || ht->second.content != prefix_content_hash(bt, block_tokens_)) break;
      ++r.host_block_count;
    }
    h = nh;
    ++r.matched_block_count;
  }
  r.matched_token_count = r.matched_block_count * block_tokens_;
  r.next_token_index = r.matched_token_count;
  r.last_block_hash = h;
  return r;
}

PrefixReservation PrefixCache::reserve_prompt(uint64_t id, const uint32_t* t, uint32_t n) {
  if (seqs_.count(id)) fail(Status::Duplicate, "PrefixCache: sequence already reserved");
  if (seqs_.size() >= max_sequences_) fail(Status::CapacityExceeded, "PrefixCache: sequence table full");
  if (n == 0) fail(Status::InvalidArgument, "PrefixCache: empty prompt");
  ++stats_.lookups;
  const PrefixLookup hit = probe_prompt(t, n);
  const uint32_t need_blocks = (n + block_tokens_ - 1) / block_tokens_;
  const uint32_t new_blocks = need_blocks - hit.matched_block_count;
  // warm blocks that the hit itself will retain cannot also be evicted for room;
  // host-tier hits need a fresh device block each
  std::vector<uint64_t> chain(hit.matched_block_count);
  uint32_t hit_warm = 0;
  {
    uint64_t h = kEmptyParentHash;
    for (uint32_t b = 0; b < hit.matched_block_count; ++b) {
      h = prefix_hash_block(t + size_t(b) * block_tokens_, block_tokens_, h);
      chain[b] = h;
      auto it = entries_.find(h);
      if (it != entries_.end() && in_lru_[it->second.block]) ++hit_warm;
    }
  }
  if (arena_.free_block_count() + lru_.size() - hit_warm < new_blocks + hit.host_block_count)
    fail(Status::CapacityExceeded, "PrefixCache: not enough KV blocks for the prompt");
  Seq s;
  s.tokens.assign(t, t + n);
  s.blocks.assign(hit.matched_block_count, kNoSlot);
  for (uint32_t b = 0; b < hit.matched_block_count; ++b)
    if (!entries_.count(chain[b])) promoting_.insert(chain[b]);
  // device hits first (retained, so promotions below cannot evict them), then promotions
  for (uint32_t b = 0; b < hit.matched_block_count; ++b) {
    auto it = entries_.find(chain[b]);
    if (it == entries_.end()) continue;
    it->second.last_used = ++clock_;
    retain(it->second.block);
    s.blocks[b] = it->second.block;
  }
  try {
    for (uint32_t b = 0; b < hit.matched_block_count; ++b) {
      if (entries_.count(chain[b])) continue;
      auto ht = host_entries_.find(chain[b]);
      const uint32_t blk = take_block();
      tier_in_.push_back(int32_t(ht->second.slot));
      tier_in_.push_back(int32_t(blk));
      host_deferred_.push_back(ht->second.slot);
      entries_.emplace(chain[b], Entry{blk, ht->second.content, ++clock_});
      block_hash_[blk] = chain[b];
      block_has_entry_[blk] = 1;
      host_lru_.erase(ht->second.lru);
      host_entries_.erase(ht);
      s.blocks[b] = blk;
      ++stats_.promoted_blocks;
    }
    promoting_.clear();
    for (uint32_t b = 0; b < new_blocks; ++b) s.blocks.push_back(take_block());
  } catch (...) {
    promoting_.clear();
    for (uint32_t b : s.blocks)
      if (b != kNoSlot) drop(b);
    throw;
  }
  s.chain = chain;
  s.committed_blocks = hit.matched_block_count;
  PrefixReservation r;
  r.sequence_id = id;
  r.requested_token_count = n;
  r.reusable_token_count = hit.matched_token_count;
  r.reserved_token_count = uint32_t(s.blocks.size()) * block_tokens_;
  r.physical_blocks = s.blocks;
  seqs_.emplace(id, std::move(s));
  ++stats_.reservations;
  if (hit.matched_block_count) ++stats_.hits;
  stats_.hit_tokens += hit.matched_token_count;
  stats_.missed_tokens += n - hit.matched_token_count;
  return r;
}

void PrefixCache::commit(uint64_t id, uint32_t computed) {
  Seq& s = seq(id);
  computed = std::min<uint32_t>(computed, (uint32_t)s.tokens.size());
  const uint32_t full = std::min<uint32_t>(computed / block_tokens_, (uint32_t)s.blocks.size());
  uint64_t h = s.chain.empty() ? kEmptyParentHash : s.chain.back();
  for (uint32_t b = s.committed_blocks; b < full; ++b) {
    const uint32_t* bt = s.tokens.data() + size_t(b) * block_tokens_;
    h = prefix_hash_block(bt, block_tokens_, h);
    s.chain.push_back(h);
    const uint32_t blk = s.blocks[b];
    auto ht = host_entries_.find(h);
    if (ht != host_entries_.end()) {  // recomputed on the device: the host copy is redundant now
      host_deferred_.push_back(ht->second.slot);
      host_lru_.erase(ht->second.lru);
      host_entries_.erase(ht);
    }
    auto it = entries_.find(h);
    if (it == entries_.end()) {
      // first publisher of this content: the entry points at our block
      if (!block_has_entry_[blk]) {
        entries_.emplace(h, Entry{blk, prefix_content_hash(bt, block_tokens_), ++clock_});
        block_hash_[blk] = h;
        block_has_entry_[blk] = 1;
        ++stats_.committed_blocks;
      }
    } else {
      it->second.last_used = ++clock_;
    }
  }
  s.committed_blocks = std::max(s.committed_blocks, full);
}

void PrefixCache::cancel_reservation(uint64_t id) {
  release_sequence(id);
  ++stats_.cancellations;
}

void PrefixCache::append_tokens(uint64_t id, const uint32_t* t, uint32_t n) {
  Seq& s = seq(id);
  s.tokens.insert(s.tokens.end(), t, t + n);
}

void PrefixCache::ensure_sequence_token_capacity(uint64_t id, uint32_t tokens) {
  Seq& s = seq(id);
  const uint32_t need = (tokens + block_tokens_ - 1) / block_tokens_;
  if (need <= s.blocks.size()) return;
  const uint32_t extra = need - (uint32_t)s.blocks.size();
  if (!can_allocate(extra)) fail(Status::CapacityExceeded, "PrefixCache: out of KV blocks");
  for (uint32_t i = 0; i < extra; ++i) s.blocks.push_back(take_block());
}

std::vector<uint32_t> PrefixCache::block_table(uint64_t id) const { return seq(id).blocks; }
const std::vector<uint32_t>& PrefixCache::block_list(uint64_t id) const { return seq(id).blocks; }
uint32_t PrefixCache::sequence_token_count(uint64_t id) const { return (uint32_t)seq(id).tokens.size(); }

void PrefixCache::release_sequence(uint64_t id) {
  auto it = seqs_.find(id);
  if (it == seqs_.end()) fail(Status::NotFound, "PrefixCache: unknown sequence");
  for (uint32_t b : it->second.blocks) drop(b);
  seqs_.erase(it);
  ++stats_.released_sequences;
}

uint32_t PrefixCache::bind_committed_prefix_from_sequence(uint64_t src, uint64_t dst, uint32_t tokens) {
  const Seq& s = seq(src);
  if (seqs_.count(dst)) fail(Status::Duplicate, "PrefixCache: destination already bound");
  const uint32_t nb = std::min<uint32_t>(tokens / block_tokens_, s.committed_blocks);
  Seq d;
  d.tokens.assign(s.tokens.begin(), s.tokens.begin() + size_t(nb) * block_tokens_);
  for (uint32_t b = 0; b < nb; ++b) {
    retain(s.blocks[b]);
    d.blocks.push_back(s.blocks[b]);
    d.chain.push_back(s.chain[b]);
  }
  d.committed_blocks = nb;
  seqs_.emplace(dst, std::move(d));
  return nb * block_tokens_;
}

}  // namespace spc
