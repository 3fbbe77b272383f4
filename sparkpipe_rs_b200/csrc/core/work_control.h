// Work control: the per-step work packets that travel between the rank that
// schedules and the ranks that execute, their transaction identity and
// payload fingerprint, the fixed MTP draft tree, execution-chunk planning, and
// the distributed KV directory.
//
// Reference: crates/spark-sched/src/work_control.rs (transaction identity and
// FNV-1a fingerprint :31-104, MTP tree :107-253, constants :293-405, queue depth
// :456-460, packets :570-780, builders :1256-1557, validation :1585-1890, KV
// directory :1896-3221). The packet is serialised in this runtime's own
// canonical little-endian layout (fixed header, optional speculative ids,
// prefill ids, lanes); the fingerprint covers exactly those bytes.
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"
#include "scheduler.h"

namespace spc {
namespace wc {

constexpr uint32_t kAbiVersion = 16;
constexpr uint32_t kPacketMagic = 0x35574350u;
constexpr uint64_t kStandaloneGeneration = 1;

// transaction phases
constexpr uint32_t kPhasePrefill = 1, kPhaseDecode = 2, kPhaseVerify = 3, kPhaseRelease = 4, kPhaseCancel = 5;
// packet flags
constexpr uint32_t kFlagPrefill = 0x01, kFlagMtpDraft = 0x02, kFlagDsparkTapCapture = 0x04,
                   kFlagDsparkSpeculativeVerify = 0x08, kFlagMtpSpeculativeVerify = 0x10,
                   kFlagReleaseSequences = 0x20, kFlagMtpResolve = 0x40, kFlagMtpTreeVerify = 0x80,
                   kFlagExecutionPayload = 0x100;
constexpr uint32_t kKnownFlags = 0x1ff;

uint64_t fingerprint_bytes(const uint8_t* data, size_t n);  // FNV-1a 64; 0 remapped to 1

struct Identity {
  uint64_t control_generation = 0, transaction_id = 0, dispatch_generation = 0, request_generation = 0,
           step_generation = 0;
  uint32_t step_chunk_index = 0, step_chunk_count = 0, transaction_phase = 0;
};
void validate_identity(const Identity& id);

// ----------------------------------------------------------------- MTP tree
// Fixed draft tree: 5 candidate tokens verified in 6 rows, depth 3.
namespace mtp {
constexpr uint32_t kCandidates = 5, kVerifierRows = 6, kExecutionSteps = 3, kMaxCommitted = 4, kContextExtension = 3;
constexpr uint32_t kResolutionNone = 0;
struct Node {
  uint8_t parent_row, depth, candidate_index, child_row_base, child_count;
};
const Node* node_at(uint32_t row);
uint32_t accepted_token_count(uint32_t path_id);
uint32_t fallback_row_index(uint32_t path_id);
uint32_t tail_candidate_index(uint32_t path_id);
uint32_t tail_parent_row_index(uint32_t path_id);
uint32_t tail_base_position_offset(uint32_t path_id);
bool resolution_is_valid(uint32_t proposed, uint32_t accepted, uint32_t path_id);
bool topology_is_valid();
struct Resolution {
  uint32_t path_id, accepted_token_count, committed_token_count, fallback_row_index;
};
// Walk the tree: at each row, follow the child whose candidate equals the verifier's token.
Resolution resolve(const uint32_t* candidates, const uint32_t* verifier_tokens, uint32_t vocab);
}  // namespace mtp

// ----------------------------------------------------------------- packets
struct Config {
  uint32_t mtp_draft_token_count = 3;
  uint32_t max_speculative_token_count = 8;
  uint32_t maximum_context_tokens = 262144;
  uint32_t kv_block_tokens = 64;
  uint32_t max_prefill_tokens_per_packet = 16384;
  uint32_t output_vocab_count = 102400;
  uint32_t max_lane_count = 1024;
  uint32_t cohort_capacity = 64;
  void validate() const;
  uint32_t kv_block_capacity() const { return maximum_context_tokens / kv_block_tokens; }
};
constexpr uint32_t queue_depth(uint32_t cohort_capacity) { return cohort_capacity + 1; }

struct Lane {
  uint64_t request_id = 0, request_generation = 0, step_generation = 0, sequence_id = 0, sequence_position = 0;
  uint32_t request_slot_index = 0, context_token_count = 0, input_token_id = 0, mtp_draft_token_count = 0;
  uint32_t speculative_token_count = 0;
  uint8_t mtp_proposed = 0, mtp_accepted = 0;
  uint16_t mtp_path_id = 0;
  std::vector<uint32_t> speculative_draft_token_ids;
};

// Execution payload (kFlagExecutionPayload): what a stage rank needs to run the
// packet's rows with no scheduler of its own, since every stage caches its layers'
// KV under the same slot numbering: each row's position and cache slot; the
// attention layout (decode: each lane's block table and context length; prefill:
// per-lane query / key offsets and, when a lane reuses cached tokens, the cache rows
// of its whole context); the rows whose logits the last stage samples; and each
// lane's sampling temperature (0 = greedy) and noise key.
struct ExecPayload {
  std::vector<int32_t> positions, slots;
  std::vector<int32_t> block_table, context_lens;
  uint32_t block_table_cols = 0;
  std::vector<int32_t> cu_q, cu_k, ctx_slots, logits_rows;
  uint32_t max_q = 0;
  std::vector<float> temperature;
  std::vector<uint64_t> sample_keys;
};

struct Packet {
  uint32_t magic = kPacketMagic, abi_version = kAbiVersion, flags = 0;
  Identity identity;
  uint64_t request_id = 0, sequence_id = 0, sequence_position = 0, deadline_time_ns = 0;
  uint32_t active_sequence_count = 0, new_token_count = 0, pipeline_slot = 0, priority = 0;
  uint32_t block_token_count = 0, max_blocks_per_sequence = 0, mtp_draft_token_count = 0;
  uint32_t rows_per_lane = 1, execution_row_count = 0, execution_batch_bucket = 0;
  std::vector<uint32_t> prefill_token_ids;
  std::vector<Lane> lanes;
  ExecPayload exec;  // serialized only with kFlagExecutionPayload
};

std::vector<uint8_t> serialize(const Packet& p);
Packet deserialize(const uint8_t* data, size_t n);
uint64_t fingerprint(const Packet& p);
void validate_packet(const Packet& p, const Config& cfg);

uint32_t select_batch_bucket(uint32_t active_sequences);  // 16 .. 1024
// (sequences per chunk, chunk count) for `rows_per_sequence` rows each under a row capacity
std::pair<uint32_t, uint32_t> execution_chunk_shape(uint32_t sequences, uint32_t rows_per_sequence,
                                                    uint32_t row_capacity, uint32_t max_bucket);

// Builds the packet of one scheduler step (decode lanes, or the prefill tokens of its sequences).
Packet build_step_packet(const StepPlan& plan, const Identity& id, const Config& cfg, uint32_t pipeline_slot);
// Splits one prefill or decode step into `chunks` micro-batch packets of contiguous
// lanes (transaction ids base.transaction_id + k, chunk k of n), each with its
// execution payload. temps / keys: per-lane sampling parameters (null: greedy).
std::vector<Packet> build_stage_packets(const StepPlan& plan, const Identity& base, const Config& cfg,
                                        uint32_t chunks, const float* temps, const uint64_t* keys);

// ----------------------------------------------------------------- KV directory
enum class KvEntryState : uint8_t { Missing = 0, InFlight = 1, Resident = 2, Transient = 3 };
enum class KvResidency : uint8_t { Gpu = 1, Nvme = 2 };

struct KvKey {
  uint64_t sequence_id;
  uint32_t logical_block;
  bool operator==(const KvKey& o) const { return sequence_id == o.sequence_id && logical_block == o.logical_block; }
};

struct KvDirectoryEntry {
  KvKey key;
  uint32_t physical_block;
  KvEntryState state;
  KvResidency residency;
  uint32_t pins;
  uint64_t content_key;  // 0 = private
  uint8_t referenced;    // clock bit
};

// Open-addressed (sequence, logical block) -> physical block map over a fixed
// pool of physical blocks: clock-sweep acquisition that skips pinned and
// in-flight entries, content-key sharing of identical blocks, pins, NVMe
// residency, and generation reset.
class KvDirectory {
 public:
  KvDirectory(uint32_t capacity_entries, uint32_t physical_blocks);
  // Maps the key to a physical block (existing, shared by content key, or a
  // fresh / swept block). Returns the physical block; *was_hit tells whether data is already there.
  uint32_t acquire(const KvKey& k, uint64_t content_key, bool* was_hit);
  const KvDirectoryEntry* find(const KvKey& k) const;
  void mark_resident(const KvKey& k);
  void mark_in_flight(const KvKey& k);
  void set_residency(const KvKey& k, KvResidency r);
  void pin(const KvKey& k);
  void unpin(const KvKey& k);
  void release_sequence(uint64_t sequence_id);
  void reset();
  uint64_t generation() const { return generation_; }
  uint32_t live_entries() const { return live_; }
  uint32_t free_blocks() const { return (uint32_t)free_blocks_.size(); }
  uint64_t sweeps() const { return sweeps_; }
  uint64_t shared_hits() const { return shared_; }

 private:
  size_t slot_of(const KvKey& k) const;
  int64_t lookup(const KvKey& k) const;
  void erase_slot(size_t s);
  uint32_t sweep_victim();
  std::vector<KvDirectoryEntry> table_;
  std::vector<uint8_t> used_;
  std::vector<uint32_t> free_blocks_;
  std::vector<int64_t> block_owner_;  // physical block -> table slot (-1 = free)
  std::vector<uint32_t> block_refs_;
  uint32_t hand_ = 0, live_ = 0, physical_;
  uint64_t generation_ = 1, sweeps_ = 0, shared_ = 0;
};

}  // namespace wc
}  // namespace spc
