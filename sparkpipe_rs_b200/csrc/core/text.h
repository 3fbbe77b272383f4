// Text plane: byte-level BPE tokenizer and chat templates.
//
// Tokenizer: loads a Hugging Face tokenizer.json (BPE model: vocab, merges,
// unk token; added tokens, the special ones matched longest-first), splits
// text into pieces with the GPT-2 byte-class rules (letters / digits / other /
// whitespace runs, an optional leading space, contractions 's 't 'm 'd 're
// 've 'll), maps piece bytes through the byte-to-unicode alphabet, and merges
// with a rank-ordered min-heap over a linked symbol list. Encoded pieces are
// memoised in a bounded cache; batches are encoded on worker threads, each
// with its own cache. A compact binary format stores a loaded tokenizer.
//
// Reference behaviour: crates/spark-text/src/tokenizer.rs:1-41 (design),
// :1192-1310 (byte classes and piece boundaries), :795 (tokenizer.json),
// :1084-1180 (compiled format), :1825 (batch encode); chat templates
// crates/spark-text/src/chat_template.rs:25-215.
#pragma once

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace spc {

class Tokenizer {
 public:
  static std::shared_ptr<Tokenizer> from_hf_json(const std::string& json_text);
  static std::shared_ptr<Tokenizer> from_compiled(const std::string& bytes);
  std::string to_compiled() const;

  std::vector<uint32_t> encode(const std::string& text, bool allow_special = true) const;
  std::vector<std::vector<uint32_t>> encode_batch(const std::vector<std::string>& texts, int workers,
                                                  bool allow_special = true) const;
  std::string decode(const std::vector<uint32_t>& ids, bool skip_special = false) const;
  std::string token_bytes(uint32_t id) const;  // raw bytes of one token

  uint32_t vocab_size() const { return (uint32_t)id_bytes_.size(); }
  int64_t token_to_id(const std::string& token) const;  // byte-level token string; -1 if absent
  bool is_special(uint32_t id) const;
  int64_t unk_id() const { return unk_; }
  uint64_t cache_hits() const { return hits_.load(std::memory_order_relaxed); }
  uint64_t cache_misses() const { return misses_.load(std::memory_order_relaxed); }

  // piece boundaries of `text` (start, length) with the GPT-2 byte classes
  static std::vector<std::pair<uint32_t, uint32_t>> split_pieces(const std::string& text);

 private:
  struct Special {
    std::string text;
    uint32_t id;
  };
  struct Merge {
    uint32_t rank;
    uint32_t merged;
  };
  using Cache = std::unordered_map<std::string, std::vector<uint32_t>>;
  void finish_load();
  void encode_piece(const char* p, size_t n, std::vector<uint32_t>& out, Cache* cache) const;
  void encode_text(const std::string& text, bool allow_special, std::vector<uint32_t>& out, Cache* cache) const;

  std::unordered_map<std::string, uint32_t> vocab_;  // byte-level token string -> id
  std::vector<std::string> id_tokens_;               // id -> byte-level token string
  std::vector<std::string> id_bytes_;                // id -> raw bytes
  std::unordered_map<uint64_t, Merge> merges_;       // (left << 32 | right) -> rank, merged id
  std::vector<std::pair<std::string, std::string>> merge_list_;
  std::vector<Special> specials_;                    // longest first
  std::vector<uint8_t> special_mask_;
  int64_t byte_token_[256];                          // id of each single-byte token, -1 if absent
  int64_t unk_ = -1;
  mutable Cache cache_;
  mutable std::mutex cache_mu_;
  // statistics, bumped by every encode thread of a batch
  mutable std::atomic<uint64_t> hits_{0}, misses_{0};
  static constexpr size_t kCacheCap = 16384;
};

// Chat templates. Styles: "glm" ([gMASK]<sop> prefix, <|system|> / <|user|> /
// <|assistant|> / <|observation|> role tags, reasoning-effort system line and
// <think> blocks) and "deepseek" (<｜begin▁of▁sentence｜>, <｜User｜>, <｜Assistant｜>).
struct ChatMessage {
  std::string role;  // system | user | assistant | tool
  std::string content;
};
constexpr uint32_t kChatAddGenerationPrompt = 0x1;
constexpr uint32_t kChatEnableThinking = 0x2;

// Incremental template writer: begin, then per message begin_message / append
// (any number of pieces: text parts, folded file attachments) / end_message,
// free text between messages, finish. Every append is checked against the
// byte capacity (CapacityExceeded). Reference: ChatTemplateWriter
// (crates/spark-text/src/chat_template.rs:76-215).
class ChatWriter {
 public:
  ChatWriter(const std::string& style, size_t capacity);
  void begin(const std::string& reasoning_effort, uint32_t flags);
  void begin_message(const std::string& role);
  void end_message(const std::string& role);
  void append(const std::string& s);
  void finish(uint32_t flags);
  const std::string& text() const { return out_; }
  size_t capacity() const { return cap_; }

 private:
  bool glm_;
  size_t cap_;
  std::string out_;
};

std::string render_chat(const std::vector<ChatMessage>& messages, const std::string& style, uint32_t flags,
                        const std::string& reasoning_effort, size_t capacity);

}  // namespace spc
