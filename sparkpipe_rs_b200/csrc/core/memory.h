// Host-side memory bookkeeping of the serving runtime:
//
//   KvArena            paged KV block arena (reference counts, residency, LRU trim)
//   Arena              size-class slab allocator with generation-checked handles
//   StatePool          fixed-slot recurrent-state pool
//   BatchSequenceTable admission / tool-exchange lifecycle of batch sequences
//   row_allocator_assign  speculative-row budget split by marginal value
//
// Behavioural contract taken from the reference's spark-core crate
// (crates/spark-core/src/kv_arena.rs:1-61, arena.rs:12-239, state_pool.rs:1-121,
// batch_sequence_table.rs:1-304, row_allocator.rs:1-159). The data structures
// are this runtime's own: free-block bitsets (lowest free block in O(n/64)),
// and a max-heap for the row allocator.
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"

namespace spc {

// ============================================================== KvArena
constexpr uint32_t kNoBlock = 0xffffffffu;
constexpr uint32_t kBlockAllocated = 0x1;
constexpr uint32_t kBlockResident = 0x2;
constexpr uint32_t kKvMaxBlockTokens = 256;
constexpr uint32_t kKvMaxLayers = 256;

struct KvArenaConfig {
  uint32_t physical_block_count = 0;
  uint32_t block_token_count = 0;
  uint32_t resident_block_capacity = 0;  // 0 = every block may be resident
  uint32_t layer_count = 1;
  uint32_t kv_head_count = 1;
  uint32_t head_dim = 1;
  uint32_t bytes_per_scalar = 2;
  uint64_t key_block_stride_bytes = 0;    // 0 = tokens * layers * heads * dim * bytes
  uint64_t value_block_stride_bytes = 0;
  uint64_t key_device_base = 0;           // opaque device addresses (never dereferenced)
  uint64_t value_device_base = 0;
};

struct KvBlockView {
  uint32_t physical_block_index;
  uint32_t token_capacity;
  uint32_t layer_count, kv_head_count, head_dim, bytes_per_scalar;
  uint64_t generation;
  uint64_t key_block_stride_bytes, value_block_stride_bytes;
  uint64_t key_device_address, value_device_address;
};

class KvArena {
 public:
  explicit KvArena(const KvArenaConfig& cfg);

  uint32_t acquire_block();
  void recycle_block(uint32_t b);
  void retain_block(uint32_t b);
  void release_block_reference(uint32_t b);
  void mark_block_resident(uint32_t b);
  void mark_block_nonresident(uint32_t b);
  void free_block(uint32_t b);
  KvBlockView resolve_block(uint32_t b) const;
  // Evict residents (lowest refcount, then oldest epoch; protected skipped) until
  // at most `target` remain; CapacityExceeded when no victim is left.
  uint32_t trim_resident_blocks(const std::vector<uint32_t>& protected_blocks, uint32_t target);
  // Same, but stops quietly when no victim is left.
  uint32_t evict_resident_blocks_to_limit(uint32_t max_resident, const std::vector<uint32_t>& protected_blocks);
  void reset();

  bool is_allocated(uint32_t b) const { return b < n_ && (blocks_[b].flags & kBlockAllocated); }
  bool is_resident(uint32_t b) const { return b < n_ && (blocks_[b].flags & kBlockResident); }
  uint32_t reference_count(uint32_t b) const { return b < n_ ? blocks_[b].refs : 0; }
  uint64_t generation(uint32_t b) const { return b < n_ ? blocks_[b].generation : 0; }
  uint64_t last_used_epoch(uint32_t b) const { return b < n_ ? blocks_[b].epoch : 0; }
  uint64_t key_device_address(uint32_t b) const { return b < n_ ? blocks_[b].key_addr : 0; }
  uint64_t value_device_address(uint32_t b) const { return b < n_ ? blocks_[b].value_addr : 0; }
  uint32_t block_token_capacity(uint32_t b) const { return b < n_ ? block_tokens_ : 0; }
  uint32_t block_token_count() const { return block_tokens_; }
  uint32_t physical_block_count() const { return n_; }
  uint32_t free_block_count() const { return free_count_; }
  uint32_t resident_block_capacity() const { return resident_cap_; }

  // counters
  uint64_t epoch() const { return epoch_; }
  uint64_t allocated_block_count() const { return allocated_; }
  uint64_t recycled_block_count() const { return recycled_; }
  uint64_t resident_block_count() const { return resident_; }
  uint64_t resident_evicted_block_count() const { return evicted_; }
  uint64_t resident_capacity_stall_count() const { return stalls_; }
  uint64_t retained_block_count() const { return retained_; }
  uint64_t released_reference_count() const { return released_; }
  uint64_t key_block_stride_bytes() const { return key_stride_; }
  uint64_t value_block_stride_bytes() const { return value_stride_; }

 private:
  struct Block {
    uint32_t flags = 0;
    uint32_t refs = 0;
    uint64_t generation = 0;
    uint64_t epoch = 0;
    uint64_t key_addr = 0;
    uint64_t value_addr = 0;
  };
  Block& checked(uint32_t b);
  Block fresh(uint32_t b) const;
  void set_free_bit(uint32_t b, bool free);
  uint32_t pick_victim(const std::vector<uint32_t>& protected_blocks) const;
  void make_room(uint32_t b);
  uint32_t trim_inner(const std::vector<uint32_t>& protected_blocks, uint32_t target);

  uint32_t n_, block_tokens_, resident_cap_, layers_, heads_, dim_, bytes_;
  uint64_t key_stride_, value_stride_, key_base_, value_base_;
  std::vector<Block> blocks_;
  std::vector<uint64_t> free_bits_;  // bit set = block free
  uint32_t free_count_ = 0;
  uint64_t epoch_ = 0, allocated_ = 0, recycled_ = 0, resident_ = 0, evicted_ = 0, stalls_ = 0, retained_ = 0,
           released_ = 0;
};

// ============================================================== Arena
struct ArenaClass {
  uint32_t slot_bytes;
  uint32_t slot_count;
};
struct ArenaHandle {
  uint32_t class_index = 0;
  uint32_t slot_index = 0;
  uint64_t generation = 0;
};

class Arena {
 public:
  static constexpr uint32_t kMaxClasses = 8;
  static constexpr uint32_t kAlignment = 16;
  explicit Arena(const std::vector<ArenaClass>& classes);
  ArenaHandle acquire(uint32_t bytes);   // smallest class that fits; throws CapacityExceeded when exhausted
  void release(const ArenaHandle& h);    // stale / foreign handles throw NotFound
  uint8_t* get(const ArenaHandle& h);    // nullptr for stale handles
  uint64_t reserved_bytes() const { return backing_.size(); }
  uint32_t class_free_count(uint32_t c) const { return c < classes_.size() ? classes_[c].free_count : 0; }
  uint64_t class_generation(uint32_t c) const { return c < classes_.size() ? classes_[c].generation : 0; }
  uint32_t class_slot_bytes(uint32_t c) const { return c < classes_.size() ? classes_[c].slot_bytes : 0; }

 private:
  struct Cls {
    uint32_t slot_bytes, slot_count;
    size_t offset;
    std::vector<uint32_t> next;  // free list links; kInUse marks an acquired slot
    std::vector<uint64_t> gen;
    uint32_t head, free_count;
    uint64_t generation;
  };
  bool live(const ArenaHandle& h) const;
  std::vector<uint8_t> backing_;
  std::vector<Cls> classes_;
};

// ============================================================== StatePool
class StatePool {
 public:
  StatePool(uint32_t slot_count, uint64_t slot_bytes);
  int64_t acquire();                 // slot index, or -1 when full
  void release(uint32_t slot);       // throws NotFound on double release / foreign slot
  bool in_use(uint32_t slot) const;
  uint8_t* slot(uint32_t slot);      // nullptr when not in use
  uint32_t free_count() const { return free_count_; }
  uint32_t slot_count() const { return (uint32_t)next_.size(); }
  uint64_t slot_bytes() const { return slot_bytes_; }

 private:
  std::vector<uint8_t> backing_;
  uint64_t slot_bytes_;
  std::vector<uint32_t> next_;
  uint32_t head_, free_count_;
};

// ============================================================== BatchSequenceTable
enum class SeqState : uint32_t { Free = 0, Active = 1, AwaitingTool = 2, Complete = 3 };

struct BatchSequence {
  uint64_t sequence_id = 0;
  SeqState state = SeqState::Free;
  uint32_t lane_count = 0;
  uint32_t exchange_number = 0;
  uint32_t context_tokens = 0;
  uint32_t fragment_base = 0;
  uint32_t fragment_count = 0;
  uint32_t generation = 0;
  uint32_t free_next = 0xffffffffu;
};

class BatchSequenceTable {
 public:
  static constexpr uint32_t kMaxSequences = 16384;
  static constexpr uint32_t kIndexBits = 14;  // handle = index | generation << 14
  BatchSequenceTable(uint32_t capacity, uint32_t lane_count);
  uint32_t admit(uint64_t sequence_id, uint32_t context_tokens, uint32_t fragment_base, uint32_t fragment_count);
  void begin_exchange(uint32_t handle, uint32_t appended_context_tokens);
  void pause_for_tool(uint32_t handle);
  void complete(uint32_t handle);
  const BatchSequence& sequence(uint32_t handle) const;
  // Expert-queue firing threshold: active * lanes * topk / experts, clamped to [1, cap].
  uint32_t firing_threshold(uint32_t topk, uint32_t expert_count, uint32_t cap) const;
  uint32_t active_count() const { return active_; }
  uint32_t awaiting_tool_count() const { return awaiting_; }
  uint32_t complete_count() const { return complete_; }
  uint64_t exchange_count() const { return exchanges_; }
  uint32_t capacity() const { return cap_; }

 private:
  uint32_t resolve(uint32_t handle) const;
  uint32_t cap_, lanes_;
  uint32_t active_ = 0, awaiting_ = 0, complete_ = 0;
  uint32_t free_head_ = 0xffffffffu, high_water_ = 0;
  uint64_t exchanges_ = 0;
  std::vector<BatchSequence> seqs_;
};

// ============================================================== row allocator
struct RowSlot {
  uint32_t commit_ema_milli;     // committed tokens per verify, x1000
  uint32_t maximum_draft_depth;  // 0 = speculation suppressed
  uint32_t probe;                // != 0: grant the fixed probe rows only
};
// Splits `firing_row_cap` rows of one wave between one real row per slot and
// speculative draft rows; draft rows go to the highest marginal value
// alpha^depth (alpha = 1 - 1000/commit_ema, milli fixed point, floor at every
// step), probes first, lower slot index on ties. Returns the total rows used.
uint32_t row_allocator_assign(const std::vector<RowSlot>& slots, uint32_t firing_row_cap,
                              uint32_t spec_row_relative_cost_milli, std::vector<uint32_t>& draft_budgets);

}  // namespace spc
