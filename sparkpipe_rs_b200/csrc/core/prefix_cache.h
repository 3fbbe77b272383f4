// Content-addressed prefix cache over the paged KV arena.
//
// Every full block of a sequence's tokens is identified by a parent-chained
// hash (block i hashes its tokens onto the hash of block i-1, starting from the
// empty-prefix hash), so two prompts that share a prefix hit the same blocks.
// The chain hash uses the same mixing and constants as the reference
// (crates/spark-core/src/prefix_cache.rs:83-157) so hash values are
// interchangeable with it; a second, position-salted content hash guards
// against chain-hash collisions.
//
// Ownership: the KvArena reference count is the only ownership record. Every
// sequence holding a block retains it once. A committed full block keeps its
// cache entry after the last sequence lets go: it stays allocated ("warm") on
// an LRU list and is freed only when an allocation needs room. Partial (last)
// blocks are private to their sequence and freed with it. Reuse of a prompt is
// capped one token short of its length so the final prompt token is always
// computed (its logits start decoding) and shared blocks are never written.
//
// Reference behaviour: probe / reserve / commit / cancel / ensure capacity /
// block table / release (crates/spark-core/src/prefix_cache.rs:879-1867).
#pragma once

#include <cstdint>
#include <list>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "common.h"
#include "memory.h"

namespace spc {

constexpr uint64_t kEmptyParentHash = 1469598103934665603ull;
constexpr uint32_t kPrefixMaxBlockTokens = 256;

uint64_t prefix_hash_block(const uint32_t* tokens, uint32_t n, uint64_t parent_hash);
uint64_t prefix_content_hash(const uint32_t* tokens, uint32_t n);

struct PromptHash {
  uint32_t token_count = 0, hashed_token_count = 0, block_count = 0, last_block_token_count = 0;
  uint64_t parent_hash = 0, prompt_hash = 0;
};
PromptHash prefix_hash_prompt(uint32_t block_tokens, uint64_t parent_hash, const uint32_t* tokens, uint32_t n);

struct PrefixLookup {
  uint32_t requested_token_count = 0;
  uint32_t matched_token_count = 0;
  uint32_t matched_block_count = 0;
  uint32_t host_block_count = 0;  // matched blocks that sit in the host tier
  uint32_t next_token_index = 0;
  uint64_t last_block_hash = kEmptyParentHash;
};

struct PrefixReservation {
  uint64_t sequence_id = 0;
  uint32_t requested_token_count = 0;
  uint32_t reusable_token_count = 0;  // prompt tokens served from cached blocks
  uint32_t reserved_token_count = 0;  // tokens the block list can hold
  std::vector<uint32_t> physical_blocks;
};

struct PrefixCacheStats {
  uint64_t lookups = 0, hits = 0, hit_tokens = 0, missed_tokens = 0;
  uint64_t committed_blocks = 0, evicted_blocks = 0, reservations = 0, cancellations = 0;
  uint64_t released_sequences = 0;
  uint64_t lookahead_protections = 0, protected_evictions = 0, trimmed_blocks = 0;
  uint64_t demoted_blocks = 0, promoted_blocks = 0, host_dropped_blocks = 0;
};

class PrefixCache {
 public:
  PrefixCache(uint32_t block_tokens, uint32_t physical_blocks, uint32_t max_sequences);

  // Longest cached prefix of `tokens`, in whole blocks, capped at n - 1 tokens.
  PrefixLookup probe_prompt(const uint32_t* tokens, uint32_t n) const;
  // Binds the cached prefix of the prompt to `seq` and allocates blocks for the
  // remaining prompt tokens (evicting warm blocks as needed). All-or-nothing:
  // on CapacityExceeded nothing stays bound.
  PrefixReservation reserve_prompt(uint64_t seq, const uint32_t* tokens, uint32_t n);
  // The sequence computed (and wrote KV for) its first `computed` tokens:
  // publishes every full block inside that range as reusable.
  void commit(uint64_t seq, uint32_t computed);
  // Rolls a reservation back (same as releasing the sequence).
  void cancel_reservation(uint64_t seq);
  // Records generated tokens of a sequence (so full decode blocks can be committed).
  void append_tokens(uint64_t seq, const uint32_t* tokens, uint32_t n);
  // Grows the block list of `seq` to hold `tokens` tokens.
  void ensure_sequence_token_capacity(uint64_t seq, uint32_t tokens);
  // Can `extra_blocks` more blocks be obtained (free or evictable)?
  bool can_allocate(uint32_t extra_blocks) const;
  std::vector<uint32_t> block_table(uint64_t seq) const;
  const std::vector<uint32_t>& block_list(uint64_t seq) const;
  uint32_t sequence_token_count(uint64_t seq) const;
  bool has_sequence(uint64_t seq) const { return seqs_.count(seq) != 0; }
  void release_sequence(uint64_t seq);
  // Evicts warm (unreferenced, committed) blocks, oldest first, until `free_blocks` are free.
  uint32_t evict_to_free(uint32_t free_blocks);
  // Lookahead protection: a queued prompt marks the cached blocks it will reuse for
  // the current epoch with a demand weight (its priority). Eviction takes unprotected
  // warm blocks first, oldest first, and protected ones last, lowest demand (then
  // fewest requesters, then oldest) first. A new epoch clears every mark.
  void reset_lookahead_protection();
  uint32_t protect_prompt_lookahead(const uint32_t* tokens, uint32_t n, uint32_t weight);  // blocks marked
  uint32_t protected_warm_blocks() const;
  // Leading chain hashes (block 0, 1, ...) that have a cache entry: a prompt's cached
  // prefix in blocks, from hashes its caller keeps (no content check).
  uint32_t cached_prefix_blocks(const std::vector<uint64_t>& chain_hashes) const;
  // Evicts warm blocks in that order until at most `max_warm` stay warm; returns how many.
  uint32_t trim_warm_blocks(uint32_t max_warm);
  // Host tier: a warm block that eviction takes is demoted to a host slot (its entry
  // stays findable) instead of being dropped, and a prompt that hits it gets a fresh
  // device block with the slot copied back (promotion). Demotions and promotions are
  // data copies the caller issues before the next step, all copies out before all
  // copies in: (device block, host slot) pairs out, (host slot, device block) pairs
  // in. A slot read by a promotion is handed out again only after the next
  // release_deferred_slots(), so a later copy out cannot overwrite it first. When the
  // host slots are all taken, the oldest host entry is dropped.
  void enable_host_tier(uint32_t first_slot, uint32_t slots);
  void take_tier_copies(std::vector<int32_t>& out, std::vector<int32_t>& in);
  bool has_tier_copies() const { return !tier_out_.empty() || !tier_in_.empty(); }
  void release_deferred_slots();
  uint32_t host_entries() const { return (uint32_t)host_entries_.size(); }
  // Binds the committed prefix of `src` (first `tokens` tokens, whole blocks) to a new sequence `dst`.
  uint32_t bind_committed_prefix_from_sequence(uint64_t src, uint64_t dst, uint32_t tokens);
  void reset();

  uint32_t block_tokens() const { return block_tokens_; }
  uint32_t free_blocks() const { return arena_.free_block_count(); }
  uint32_t warm_blocks() const { return (uint32_t)lru_.size(); }
  uint32_t entry_count() const { return (uint32_t)entries_.size(); }
  uint32_t sequence_count() const { return (uint32_t)seqs_.size(); }
  const PrefixCacheStats& stats() const { return stats_; }
  const KvArena& arena() const { return arena_; }

 private:
  struct Entry {
    uint32_t block;
    uint64_t content;
    uint64_t last_used;
    uint64_t protect_epoch = 0;
    uint32_t protect_weight = 0, protect_count = 0;
  };
  uint32_t evict_one();  // frees the warm block that eviction order picks; returns it
  struct Seq {
    std::vector<uint32_t> tokens;   // prompt + generated tokens known so far
    std::vector<uint32_t> blocks;
    std::vector<uint64_t> chain;    // chain hash of each committed full block
    uint32_t committed_blocks = 0;  // leading blocks published as reusable
  };
  uint32_t take_block();
  void retain(uint32_t b);
  void drop(uint32_t b);
  Seq& seq(uint64_t id);
  const Seq& seq(uint64_t id) const;

  uint32_t block_tokens_;
  uint32_t max_sequences_;
  KvArena arena_;
  std::unordered_map<uint64_t, Entry> entries_;      // chain hash -> entry
  std::vector<uint64_t> block_hash_;                 // block -> chain hash of its entry (0 = none)
  std::vector<uint8_t> block_has_entry_;
  std::list<uint32_t> lru_;                          // warm blocks, oldest first
  std::vector<std::list<uint32_t>::iterator> lru_pos_;
  std::vector<uint8_t> in_lru_;
  std::unordered_map<uint64_t, Seq> seqs_;
  uint64_t clock_ = 0;
  uint64_t protect_epoch_ = 1;
  PrefixCacheStats stats_;
  // host tier
  struct HostEntry {
    uint32_t slot;
    uint64_t content;
    std::list<uint64_t>::iterator lru;
  };
  bool host_enabled_ = false;
  std::unordered_map<uint64_t, HostEntry> host_entries_;  // chain hash -> host slot
  std::list<uint64_t> host_lru_;                           // chain hashes, oldest first
  std::vector<uint32_t> host_free_, host_deferred_;
  std::vector<int32_t> tier_out_, tier_in_;
  std::unordered_set<uint64_t> promoting_;  // host entries a reservation is bringing back
  static constexpr uint32_t kNoSlot = 0xffffffffu;
  // a free slot, dropping the oldest host entry not being promoted when none is free; kNoSlot if none
  uint32_t host_slot();
};

}  // namespace spc
