#include "text.h"

#include <algorithm>
#include <cstring>
#include <queue>
#include <thread>

#include "json.h"

namespace spc {

namespace {

// GPT-2 byte-to-unicode alphabet: printable bytes map to themselves, the rest
// to U+0100 onwards in byte order.
struct ByteAlphabet {
  uint32_t to_cp[256];
  std::unordered_map<uint32_t, uint8_t> to_byte;
  ByteAlphabet() {
    uint32_t next = 256;
    for (int b = 0; b < 256; ++b) {
      const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
      to_cp[b] = keep ? uint32_t(b) : next++;
      to_byte[to_cp[b]] = uint8_t(b);
    }
  }
};
const ByteAlphabet& alphabet() {
  static ByteAlphabet a;
  return a;
}

void put_utf8(std::string& o, uint32_t cp) {
  if (cp < 0x80) o += char(cp);
  else if (cp < 0x800) { o += char(0xC0 | (cp >> 6)); o += char(0x80 | (cp & 0x3F)); }
  else { o += char(0xE0 | (cp >> 12)); o += char(0x80 | ((cp >> 6) & 0x3F)); o += char(0x80 | (cp & 0x3F)); }
}

// byte-level token string -> raw bytes (each UTF-8 codepoint is one byte)
bool token_to_bytes(const std::string& tok, std::string& out) {
  const auto& A = alphabet();
  out.clear();
  for (size_t i = 0; i < tok.size();) {
    const unsigned char c = tok[i];
    uint32_t cp;
    int n;
    if (c < 0x80) { cp = c; n = 1; }
    else if ((c >> 5) == 6) { cp = c & 0x1F; n = 2; }
    else if ((c >> 4) == 14) { cp = c & 0x0F; n = 3; }
    else { cp = c & 0x07; n = 4; }
    if (i + n > tok.size()) return false;
    for (int k = 1; k < n; ++k) cp = (cp << 6) | (tok[i + k] & 0x3F);
    i += n;
    auto it = A.to_byte.find(cp);
    if (it == A.to_byte.end()) return false;
    out += char(it->second);
  }
  return true;
}

// piece boundary rules: 1 whitespace, 2 letter (or any byte >= 0x80), 3 digit, 4 other
uint8_t byte_class(unsigned char b) {
  if (b == ' ' || (b >= 9 && b <= 13)) return 1;
  if (b >= 0x80 || (b >= 'a' && b <= 'z') || (b >= 'A' && b <= 'Z')) return 2;
  if (b >= '0' && b <= '9') return 3;
  return 4;
}
bool ascii_ws(unsigned char b) { return b == ' ' || b == '\t' || b == '\n' || b == '\r' || b == 0x0b || b == 0x0c; }
size_t contraction(const std::string& t, size_t i) {
  if (i + 1 >= t.size() || t[i] != '\'') return 0;
  const char a = char(std::tolower((unsigned char)t[i + 1]));
  if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
  if (i + 2 >= t.size()) return 0;
  const char b = char(std::tolower((unsigned char)t[i + 2]));
  if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
  return 0;
}
size_t run_end(const std::string& t, size_t i, uint8_t cls, bool stop_at_contraction) {
  while (i < t.size() && byte_class((unsigned char)t[i]) == cls) {
    if (stop_at_contraction && contraction(t, i)) break;
    ++i;
  }
  return i;
}

}  // namespace

std::vector<std::pair<uint32_t, uint32_t>> Tokenizer::split_pieces(const std::string& t) {
  std::vector<std::pair<uint32_t, uint32_t>> out;
  size_t i = 0;
  while (i < t.size()) {
    size_t n = contraction(t, i);
    if (!n) {
      if (t[i] == ' ' && i + 1 < t.size() && !ascii_ws((unsigned char)t[i + 1])) {
        const uint8_t c = byte_class((unsigned char)t[i + 1]);
        n = run_end(t, i + 1, c, c == 4) - i;
      } else {
        const uint8_t c = byte_class((unsigned char)t[i]);
        n = run_end(t, i, c, c == 4) - i;
        if (n == 0) n = 1;  // an apostrophe that starts no contraction
      }
    }
    out.emplace_back(uint32_t(i), uint32_t(n));
    i += n;
  }
  return out;
}

void Tokenizer::finish_load() {
  for (int b = 0; b < 256; ++b) {
    std::string tok;
    put_utf8(tok, alphabet().to_cp[b]);
    auto it = vocab_.find(tok);
    byte_token_[b] = it == vocab_.end() ? -1 : int64_t(it->second);
  }
  special_mask_.assign(id_bytes_.size(), 0);
  for (auto& s : specials_)
    if (s.id < special_mask_.size()) special_mask_[s.id] = 1;
  std::stable_sort(specials_.begin(), specials_.end(),
                   [](const Special& a, const Special& b) { return a.text.size() > b.text.size(); });
}

std::shared_ptr<Tokenizer> Tokenizer::from_hf_json(const std::string& text) {
  const Json root = Json::parse(text);
  const Json& model = root.at("model");
  if (const Json* ty = model.get("type"); ty && ty->str() != "BPE")
    fail(Status::SchemaError, "tokenizer: only BPE models are supported");
  auto tk = std::make_shared<Tokenizer>();
  uint32_t max_id = 0;
  for (const auto& kv : model.at("vocab").obj()) max_id = std::max<uint32_t>(max_id, uint32_t(kv.second.int64()));
  if (const Json* added = root.get("added_tokens"))
    for (const auto& a : added->arr()) max_id = std::max<uint32_t>(max_id, uint32_t(a.at("id").int64()));
  tk->id_tokens_.assign(max_id + 1, std::string());
  tk->id_bytes_.assign(max_id + 1, std::string());
  for (const auto& kv : model.at("vocab").obj()) {
    const uint32_t id = uint32_t(kv.second.int64());
    tk->vocab_[kv.first] = id;
    tk->id_tokens_[id] = kv.first;
    std::string raw;
    tk->id_bytes_[id] = token_to_bytes(kv.first, raw) ? raw : kv.first;
  }
  if (const Json* added = root.get("added_tokens")) {
    for (const auto& a : added->arr()) {
      const uint32_t id = uint32_t(a.at("id").int64());
      const std::string& content = a.at("content").str();
      tk->id_tokens_[id] = content;
      tk->id_bytes_[id] = content;
      tk->vocab_[content] = id;
      const Json* sp = a.get("special");
      if (sp && sp->boolean()) tk->specials_.push_back(Special{content, id});
    }
  }
  if (const Json* unk = model.get("unk_token"); unk && unk->is_string()) {
    auto it = tk->vocab_.find(unk->str());
    if (it != tk->vocab_.end()) tk->unk_ = it->second;
  }
  uint32_t rank = 0;
  for (const auto& m : model.at("merges").arr()) {
    std::string l, r;
    if (m.is_string()) {
      const std::string& s = m.str();
      const size_t sp = s.find(' ');
      if (sp == std::string::npos) fail(Status::SchemaError, "tokenizer: merge without a space");
      l = s.substr(0, sp);
      r = s.substr(sp + 1);
    } else {
      l = m.arr().at(0).str();
      r = m.arr().at(1).str();
    }
    tk->merge_list_.emplace_back(l, r);
    auto il = tk->vocab_.find(l), ir = tk->vocab_.find(r), im = tk->vocab_.find(l + r);
    if (il != tk->vocab_.end() && ir != tk->vocab_.end() && im != tk->vocab_.end()) {
      const uint64_t key = (uint64_t(il->second) << 32) | ir->second;
      if (!tk->merges_.count(key)) tk->merges_[key] = Merge{rank, im->second};
    }
    ++rank;
  }
  tk->finish_load();
  return tk;
}

std::string Tokenizer::to_compiled() const {
  std::string o = "SPTK";
  auto u32 = [&](uint32_t v) { char b[4]; put_u32(reinterpret_cast<uint8_t*>(b), v); o.append(b, 4); };
  auto str = [&](const std::string& s) { u32(uint32_t(s.size())); o += s; };
  u32(1);  // format version
  u32(uint32_t(id_tokens_.size()));
  for (const auto& t : id_tokens_) str(t);
  u32(uint32_t(merge_list_.size()));
  for (const auto& m : merge_list_) { str(m.first); str(m.second); }
  u32(uint32_t(specials_.size()));
  for (const auto& s : specials_) { u32(s.id); str(s.text); }
  u32(uint32_t(unk_ + 1));
  return o;
}

std::shared_ptr<Tokenizer> Tokenizer::from_compiled(const std::string& b) {
  size_t i = 0;
  auto need = [&](size_t n) { if (i + n > b.size()) fail(Status::ParseError, "tokenizer: truncated compiled file"); };
  auto u32 = [&]() { need(4); uint32_t v = get_u32(reinterpret_cast<const uint8_t*>(b.data() + i)); i += 4; return v; };
  auto str = [&]() { const uint32_t n = u32(); need(n); std::string s = b.substr(i, n); i += n; return s; };
  need(4);
  if (b.compare(0, 4, "SPTK") != 0) fail(Status::ParseError, "tokenizer: not a compiled tokenizer");
  i = 4;
  if (u32() != 1) fail(Status::AbiMismatch, "tokenizer: unknown compiled format version");
  auto tk = std::make_shared<Tokenizer>();
  const uint32_t n = u32();
  tk->id_tokens_.resize(n);
  tk->id_bytes_.resize(n);
  for (uint32_t id = 0; id < n; ++id) {
    tk->id_tokens_[id] = str();
    if (!tk->id_tokens_[id].empty()) tk->vocab_[tk->id_tokens_[id]] = id;
  }
  const uint32_t nm = u32();
  for (uint32_t r = 0; r < nm; ++r) {
    std::string l = str(), rr = str();
    tk->merge_list_.emplace_back(l, rr);
  }
  const uint32_t ns = u32();
  for (uint32_t k = 0; k < ns; ++k) {
    const uint32_t id = u32();
    tk->specials_.push_back(Special{str(), id});
  }
  tk->unk_ = int64_t(u32()) - 1;
  for (uint32_t id = 0; id < n; ++id) {
    std::string raw;
    tk->id_bytes_[id] = token_to_bytes(tk->id_tokens_[id], raw) ? raw : tk->id_tokens_[id];
  }
  for (const auto& s : tk->specials_) tk->id_bytes_[s.id] = s.text;
  uint32_t rank = 0;
  for (const auto& m : tk->merge_list_) {
    auto il = tk->vocab_.find(m.first), ir = tk->vocab_.find(m.second), im = tk->vocab_.find(m.first + m.second);
    if (il != tk->vocab_.end() && ir != tk->vocab_.end() && im != tk->vocab_.end()) {
      const uint64_t key = (uint64_t(il->second) << 32) | ir->second;
      if (!tk->merges_.count(key)) tk->merges_[key] = Merge{rank, im->second};
    }
    ++rank;
  }
  tk->finish_load();
  return tk;
}

void Tokenizer::encode_piece(const char* p, size_t n, std::vector<uint32_t>& out, Cache* cache) const {
  const std::string key(p, n);
  if (cache) {
    auto it = cache->find(key);
    if (it != cache->end()) {
      hits_.fetch_add(1, std::memory_order_relaxed);
      out.insert(out.end(), it->second.begin(), it->second.end());
      return;
    }
    misses_.fetch_add(1, std::memory_order_relaxed);
  }
  // symbols: one per byte, doubly linked; merges applied lowest rank first
  std::vector<int64_t> sym(n);
  std::vector<int> prev(n), next(n);
  for (size_t i = 0; i < n; ++i) {
    sym[i] = byte_token_[(unsigned char)p[i]];
    prev[i] = int(i) - 1;
    next[i] = i + 1 < n ? int(i + 1) : -1;
  }
  struct Cand {
    uint32_t rank;
    int left;
    int64_t a, b;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : left > o.left; }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto push = [&](int l) {
    if (l < 0) return;
    const int r = next[l];
    if (r < 0 || sym[l] < 0 || sym[r] < 0) return;
    auto it = merges_.find((uint64_t(sym[l]) << 32) | uint64_t(sym[r]));
    if (it != merges_.end()) heap.push(Cand{it->second.rank, l, sym[l], sym[r]});
  };
  for (size_t i = 0; i + 1 < n; ++i) push(int(i));
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    const int l = c.left, r = next[l];
    if (sym[l] != c.a || r < 0 || sym[r] != c.b) continue;  // stale candidate
    sym[l] = merges_.at((uint64_t(c.a) << 32) | uint64_t(c.b)).merged;
    sym[r] = -2;  // removed
    next[l] = next[r];
    if (next[r] >= 0) prev[next[r]] = l;
    push(prev[l]);
    push(l);
  }
  std::vector<uint32_t> ids;
  for (int i = n ? 0 : -1; i >= 0; i = next[i]) {
    if (sym[i] >= 0) ids.push_back(uint32_t(sym[i]));
    else if (sym[i] == -1 && unk_ >= 0) ids.push_back(uint32_t(unk_));
  }
  if (cache) {
    if (cache->size() >= kCacheCap) cache->clear();
    (*cache)[key] = ids;
  }
  out.insert(out.end(), ids.begin(), ids.end());
}

void Tokenizer::encode_text(const std::string& text, bool allow_special, std::vector<uint32_t>& out,
                            Cache* cache) const {
  size_t seg = 0;
  auto flush = [&](size_t end) {
    if (end <= seg) return;
    const std::string part = text.substr(seg, end - seg);
    for (const auto& pc : split_pieces(part)) encode_piece(part.data() + pc.first, pc.second, out, cache);
  };
  if (allow_special && !specials_.empty()) {
    for (size_t i = 0; i < text.size();) {
      bool hit = false;
      for (const auto& s : specials_) {
        if (text.compare(i, s.text.size(), s.text) == 0) {
          flush(i);
          out.push_back(s.id);
          i += s.text.size();
          seg = i;
          hit = true;
          break;
        }
      }
      if (!hit) ++i;
    }
  }
  flush(text.size());
}

std::vector<uint32_t> Tokenizer::encode(const std::string& text, bool allow_special) const {
  std::vector<uint32_t> out;
  std::lock_guard<std::mutex> lk(cache_mu_);
  encode_text(text, allow_special, out, &cache_);
  return out;
}

std::vector<std::vector<uint32_t>> Tokenizer::encode_batch(const std::vector<std::string>& texts, int workers,
                                                           bool allow_special) const {
  std::vector<std::vector<uint32_t>> out(texts.size());
  if (workers <= 1 || texts.size() < 2) {
    for (size_t i = 0; i < texts.size(); ++i) out[i] = encode(texts[i], allow_special);
    return out;
  }
  workers = std::min<int>(workers, int(texts.size()));
  std::vector<std::thread> th;
  for (int w = 0; w < workers; ++w) {
    th.emplace_back([&, w]() {
      Cache local;  // per-worker piece cache: no sharing, no locks
      for (size_t i = w; i < texts.size(); i += workers) encode_text(texts[i], allow_special, out[i], &local);
    });
  }
  for (auto& t : th) t.join();
  return out;
}

std::string Tokenizer::decode(const std::vector<uint32_t>& ids, bool skip_special) const {
  std::string o;
  for (uint32_t id : ids) {
    if (id >= id_bytes_.size()) fail(Status::InvalidArgument, "tokenizer: token id out of range");
    if (skip_special && special_mask_[id]) continue;
    o += id_bytes_[id];
  }
  return o;
}

std::string Tokenizer::token_bytes(uint32_t id) const {
  if (id >= id_bytes_.size()) fail(Status::InvalidArgument, "tokenizer: token id out of range");
  return id_bytes_[id];
}

int64_t Tokenizer::token_to_id(const std::string& token) const {
  auto it = vocab_.find(token);
  return it == vocab_.end() ? -1 : int64_t(it->second);
}

bool Tokenizer::is_special(uint32_t id) const { return id < special_mask_.size() && special_mask_[id]; }

// ------------------------------------------------------------------ chat templates
namespace {
const char* kDsBos = "<\xef\xbd\x9c" "begin\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>";
const char* kDsEos = "<\xef\xbd\x9c" "end\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>";
const char* kDsUser = "<\xef\xbd\x9cUser\xef\xbd\x9c>";
const char* kDsAssistant = "<\xef\xbd\x9c" "Assistant\xef\xbd\x9c>";
const char* kDsTool = "<\xef\xbd\x9ctool\xe2\x96\x81output\xef\xbd\x9c>";
}  // namespace

ChatWriter::ChatWriter(const std::string& style, size_t capacity) : cap_(capacity) {
  if (style == "glm") glm_ = true;
  else if (style == "deepseek") glm_ = false;
  else fail(Status::InvalidArgument, "chat: unknown template style " + style);
}

void ChatWriter::append(const std::string& s) {
  if (out_.size() + s.size() > cap_) fail(Status::CapacityExceeded, "chat: rendered prompt exceeds capacity");
  out_ += s;
}

void ChatWriter::begin(const std::string& effort, uint32_t flags) {
  if (flags & ~(kChatAddGenerationPrompt | kChatEnableThinking)) fail(Status::InvalidArgument, "chat: unknown flags");
  if (!glm_) { append(kDsBos); return; }
  append("[gMASK]<sop>");
  if (flags & kChatEnableThinking) {
    append("<|system|>Reasoning Effort: ");
    append((effort == "high" || effort == "High") ? "High" : "Max");
  }
}

void ChatWriter::begin_message(const std::string& role) {
  if (glm_) {
    if (role == "system") append("<|system|>");
    else if (role == "user") append("<|user|>");
    else if (role == "assistant") { append("<|assistant|>"); append("<think></think>"); }
    else if (role == "tool") { append("<|observation|>"); append("<tool_response>"); }
    else fail(Status::InvalidArgument, "chat: unknown role " + role);
  } else {
    if (role == "system") {}
    else if (role == "user") append(kDsUser);
    else if (role == "assistant") append(kDsAssistant);
    else if (role == "tool") append(kDsTool);
    else fail(Status::InvalidArgument, "chat: unknown role " + role);
  }
}

void ChatWriter::end_message(const std::string& role) {
  if (glm_) {
    if (role == "tool") append("</tool_response>");
  } else if (role == "assistant") {
    append(kDsEos);
  }
}

void ChatWriter::finish(uint32_t flags) {
  if (!(flags & kChatAddGenerationPrompt)) return;
  if (glm_) {
    append("<|assistant|>");
    append((flags & kChatEnableThinking) ? "<think>" : "<think></think>");
  } else {
    append(kDsAssistant);
  }
}

std::string render_chat(const std::vector<ChatMessage>& msgs, const std::string& style, uint32_t flags,
                        const std::string& effort, size_t capacity) {
  ChatWriter w(style, capacity);
  w.begin(effort, flags);
  for (const auto& m : msgs) {
    w.begin_message(m.role);
    w.append(m.content);
    w.end_message(m.role);
  }
  w.finish(flags);
  return w.text();
}

}  // namespace spc
