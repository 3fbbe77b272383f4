#include "stagepack.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

#include "json.h"

namespace spc {
namespace pack {

namespace {

inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
constexpr uint64_t kMulA = 0x9E3779B97F4A7C15ull;  // 2^64 / golden ratio
constexpr uint64_t kMulB = 0xD6E8FEB86659FD93ull;  // an odd mixing constant

uint64_t mix_final(uint64_t h) {
  h ^= h >> 33;
  h *= kMulB;
  h ^= h >> 29;
  h *= kMulA;
  h ^= h >> 32;
  return h;
}

uint64_t product(const std::vector<uint64_t>& v, size_t from = 0, size_t to = SIZE_MAX) {
  uint64_t p = 1;
  for (size_t i = from; i < std::min(to, v.size()); ++i) {
    if (v[i] != 0 && p > UINT64_MAX / v[i]) fail(Status::CapacityExceeded, "stage pack: tensor size overflow");
    p *= v[i];
  }
  return p;
}

std::string data_name(uint32_t n) {
  char b[32];
  std::snprintf(b, sizeof b, "data_%04u.bin", n);
  return b;
}

void write_all(int fd, const void* p, size_t n, const std::string& what) {
  const char* c = static_cast<const char*>(p);
  while (n) {
    const ssize_t w = ::write(fd, c, n);
    if (w < 0 && errno == EINTR) continue;
    if (w <= 0) fail(Status::IoError, "stage pack: write failed: " + what);
    c += w;
    n -= size_t(w);
  }
}

std::string read_text(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(Status::NotFound, "stage pack: no index at " + path);
  std::ostringstream s;
  s << f.rdbuf();
  return s.str();
}

}  // namespace

uint64_t fingerprint(const void* data, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  uint64_t lane[4] = {kMulA, kMulB, ~kMulA, ~kMulB};
  size_t i = 0;
  for (; i + 32 <= n; i += 32) {
    for (int k = 0; k < 4; ++k) {
      uint64_t w;
      std::memcpy(&w, p + i + 8 * k, 8);
      lane[k] = rotl(lane[k] ^ (w * kMulA), 31) * kMulB;
    }
  }
  uint64_t tail = 0;
  for (size_t j = 0; i + j < n; ++j) {
    tail = (tail << 8) | p[i + j];
    if (j % 8 == 7) tail = rotl(tail, 17) * kMulA;
  }
  uint64_t h = uint64_t(n) * kMulA;
  for (int k = 0; k < 4; ++k) h = rotl(h ^ mix_final(lane[k]), 27) * kMulB;
  return mix_final(h ^ mix_final(tail));
}

// ------------------------------------------------------------------ writer
Writer::Writer(const std::string& root, const std::string& model_id, const std::string& metadata_json)
    : root_(root), model_id_(model_id), metadata_(metadata_json.empty() ? "{}" : metadata_json) {
  if (root.empty() || root.size() + 32 >= kPathBytes) fail(Status::InvalidArgument, "stage pack: root path");
  Json::parse(metadata_);  // must be JSON (ParseError otherwise)
  if (::mkdir(root.c_str(), 0755) != 0 && errno != EEXIST) fail(Status::IoError, "stage pack: cannot create " + root);
  ::unlink((root_ + "/" + kIndexFile).c_str());  // a stale index must not describe new data
  open_next();
}

Writer::~Writer() {
  if (fd_ >= 0) ::close(fd_);
}

void Writer::open_next() {
  if (fd_ >= 0) ::close(fd_);
  const std::string path = root_ + "/" + data_name(file_no_);
  fd_ = ::open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd_ < 0) fail(Status::IoError, "stage pack: cannot create " + path);
  pos_ = 0;
}

void Writer::add(const std::string& name, const std::string& dtype, const std::vector<uint64_t>& shape,
                 uint64_t bytes_per_element, const void* data, uint64_t bytes) {
  if (finished_) fail(Status::InvalidArgument, "stage pack: the index is already written");
  if (name.empty() || dtype.empty() || shape.empty() || shape.size() > kMaxRank || bytes_per_element == 0 ||
      (bytes && !data))
    fail(Status::InvalidArgument, "stage pack: tensor " + name);
  for (const Entry& e : entries_)
    if (e.name == name) fail(Status::Duplicate, "stage pack: tensor " + name + " twice");
  if (product(shape) * bytes_per_element != bytes)
    fail(Status::SchemaError, "stage pack: " + name + " bytes disagree with its shape");
  const uint64_t start = (pos_ + kAlign - 1) / kAlign * kAlign;
  if (pos_ > 0 && start + bytes > kFileLimit) {
    ++file_no_;
    open_next();
  }
  const uint64_t at = (pos_ + kAlign - 1) / kAlign * kAlign;
  if (at > pos_) {
    static const char zeros[kAlign] = {};
    write_all(fd_, zeros, size_t(at - pos_), name);
  }
  write_all(fd_, data, size_t(bytes), name);
  Entry e;
  e.name = name;
  e.dtype = dtype;
  e.shape = shape;
  e.bytes_per_element = bytes_per_element;
  e.file = data_name(file_no_);
  e.offset = at;
  e.bytes = bytes;
  e.fingerprint = fingerprint(data, size_t(bytes));
  entries_.push_back(std::move(e));
  pos_ = at + bytes;
  total_ += bytes;
}

void Writer::finish() {
  if (finished_) return;
  if (fd_ >= 0) {
    if (::fsync(fd_) != 0) fail(Status::IoError, "stage pack: fsync");
    ::close(fd_);
    fd_ = -1;
  }
  Json idx = Json::make_object();
  idx.set("format", Json::make_string(kFormat));
  idx.set("model_id", Json::make_string(model_id_));
  idx.set("metadata", Json::parse(metadata_));
  Json tensors = Json::make_array();
  for (const Entry& e : entries_) {
    Json t = Json::make_object();
    t.set("name", Json::make_string(e.name));
    t.set("dtype", Json::make_string(e.dtype));
    Json sh = Json::make_array();
    for (uint64_t d : e.shape) sh.push(Json::make_int(int64_t(d)));
    t.set("shape", sh);
    t.set("bytes_per_element", Json::make_int(int64_t(e.bytes_per_element)));
    t.set("file", Json::make_string(e.file));
    t.set("offset", Json::make_int(int64_t(e.offset)));
    t.set("bytes", Json::make_int(int64_t(e.bytes)));
    char fp[17];
    std::snprintf(fp, sizeof fp, "%016llx", (unsigned long long)e.fingerprint);
    t.set("fingerprint", Json::make_string(fp));
    tensors.push(std::move(t));
  }
  idx.set("tensors", std::move(tensors));
  const std::string tmp = root_ + "/" + kIndexFile + ".tmp", fin = root_ + "/" + kIndexFile;
  const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd < 0) fail(Status::IoError, "stage pack: cannot write the index");
  const std::string text = idx.dump();
  write_all(fd, text.data(), text.size(), "index");
  ::fsync(fd);
  ::close(fd);
  if (::rename(tmp.c_str(), fin.c_str()) != 0) fail(Status::IoError, "stage pack: cannot publish the index");
  finished_ = true;
}

// ------------------------------------------------------------------ reader
Pack Pack::open(const std::string& root) {
  Pack p;
  p.root_ = root;
  const Json idx = Json::parse(read_text(root + "/" + kIndexFile));
  if (!idx.is_object() || idx.at("format").str() != kFormat) fail(Status::SchemaError, "stage pack: format");
  p.model_id_ = idx.at("model_id").str();
  p.metadata_ = idx.at("metadata").dump();
  std::unordered_map<std::string, uint64_t> file_size;
  for (const Json& t : idx.at("tensors").arr()) {
    Entry e;
    e.name = t.at("name").str();
    e.dtype = t.at("dtype").str();
    for (const Json& d : t.at("shape").arr()) {
      if (!d.is_integer() || d.int64() < 0) fail(Status::SchemaError, "stage pack: shape of " + e.name);
      e.shape.push_back(uint64_t(d.int64()));
    }
    const int64_t bpe = t.at("bytes_per_element").int64(), off = t.at("offset").int64(), n = t.at("bytes").int64();
    e.file = t.at("file").str();
    if (e.name.empty() || e.shape.empty() || e.shape.size() > kMaxRank || bpe <= 0 || off < 0 || n < 0 ||
        e.file.find('/') != std::string::npos || e.file.find("..") != std::string::npos)
      fail(Status::SchemaError, "stage pack: entry " + e.name);
    e.bytes_per_element = uint64_t(bpe);
    e.offset = uint64_t(off);
    e.bytes = uint64_t(n);
    if (product(e.shape) * e.bytes_per_element != e.bytes)
      fail(Status::SchemaError, "stage pack: " + e.name + " bytes disagree with its shape");
    e.fingerprint = std::stoull(t.at("fingerprint").str(), nullptr, 16);
    auto fs = file_size.find(e.file);
    if (fs == file_size.end()) {
      struct stat st{};
      if (::stat((root + "/" + e.file).c_str(), &st) != 0) fail(Status::NotFound, "stage pack: missing " + e.file);
      fs = file_size.emplace(e.file, uint64_t(st.st_size)).first;
    }
    if (e.offset + e.bytes > fs->second) fail(Status::SchemaError, "stage pack: " + e.name + " outside its file");
    if (!p.by_name_.emplace(e.name, p.entries_.size()).second) fail(Status::Duplicate, "stage pack: " + e.name);
    p.entries_.push_back(std::move(e));
  }
  return p;
}

std::vector<std::string> Pack::names() const {
  std::vector<std::string> out;
  for (const Entry& e : entries_) out.push_back(e.name);
  return out;
}

const Entry& Pack::entry(const std::string& name) const {
  auto it = by_name_.find(name);
  if (it == by_name_.end()) fail(Status::NotFound, "stage pack: no tensor " + name);
  return entries_[it->second];
}

Region Pack::resolve(const std::string& name, const std::string& dtype, const std::vector<uint64_t>& shape,
                     uint64_t bytes_per_element) const {
  const Entry& e = entry(name);
  if (e.dtype != dtype || e.shape != shape || e.bytes_per_element != bytes_per_element)
    fail(Status::SchemaError, "stage pack: " + name + " is stored with another dtype or shape");
  Region r;
  r.file_path = root_ + "/" + e.file;
  if (r.file_path.size() >= kPathBytes) fail(Status::CapacityExceeded, "stage pack: path too long");
  r.file_offset = e.offset;
  r.tensor_bytes = e.bytes;
  return r;
}

void Pack::pread_all(const Entry& e, uint64_t rel, void* dst, uint64_t n) const {
  if (rel + n > e.bytes) fail(Status::InvalidArgument, "stage pack: read past " + e.name);
  const std::string path = root_ + "/" + e.file;
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) fail(Status::IoError, "stage pack: cannot open " + path);
  char* c = static_cast<char*>(dst);
  uint64_t off = e.offset + rel;
  while (n) {
    const ssize_t r = ::pread(fd, c, size_t(std::min<uint64_t>(n, 1ull << 30)), off_t(off));
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) {
      ::close(fd);
      fail(Status::IoError, "stage pack: short read of " + e.name);
    }
    c += r;
    off += uint64_t(r);
    n -= uint64_t(r);
  }
  ::close(fd);
}

void Pack::read(const std::string& name, void* dst, uint64_t dst_bytes, bool verify) const {
  const Entry& e = entry(name);
  if (dst_bytes != e.bytes) fail(Status::InvalidArgument, "stage pack: destination is not " + name + "'s size");
  pread_all(e, 0, dst, e.bytes);
  if (verify && fingerprint(dst, size_t(e.bytes)) != e.fingerprint)
    fail(Status::HashMismatch, "stage pack: " + name + " does not match its fingerprint");
}

void Pack::read_rows(const std::string& name, uint64_t row0, uint64_t rows, void* dst, uint64_t dst_bytes) const {
  const Entry& e = entry(name);
  const uint64_t row_bytes = product(e.shape, 1) * e.bytes_per_element;
  if (row0 + rows > e.shape[0] || dst_bytes != rows * row_bytes)
    fail(Status::InvalidArgument, "stage pack: row range of " + name);
  pread_all(e, row0 * row_bytes, dst, rows * row_bytes);
}

tp::View Pack::read_shard(const std::string& name, const tp::Shape& shape, const tp::Geometry& g, void* dst,
                          uint64_t dst_bytes) const {
  const Entry& e = entry(name);
  tp::TensorSpec spec;
  spec.name = name;
  spec.dims = e.shape;
  spec.element_bytes = uint32_t(e.bytes_per_element);
  const tp::View v = tp::compute_view(spec, shape, g);
  if (v.shard_class == tp::ShardClass::Replicated) {
    if (dst_bytes != e.bytes) fail(Status::InvalidArgument, "stage pack: destination is not " + name + "'s size");
    pread_all(e, 0, dst, e.bytes);
    return v;
  }
  if (dst_bytes != v.shard_bytes) fail(Status::InvalidArgument, "stage pack: destination is not the shard's size");
  const uint32_t d = v.split_dimension;
  const uint64_t inner = product(e.shape, d + 1) * e.bytes_per_element;  // bytes of one index of dim d
  const uint64_t outer = product(e.shape, 0, d);
  const uint64_t pitch = e.shape[d] * inner;                             // one outer row in the file
  char* out = static_cast<char*>(dst);
  if (d == 0) {  // each part is one contiguous range
    for (const auto& r : v.ranges) {
      pread_all(e, r.first * inner, out, r.second * inner);
      out += r.second * inner;
    }
    return v;
  }
  for (uint64_t o = 0; o < outer; ++o)  // inner split: one chunk per part per outer row
    for (const auto& r : v.ranges) {
      pread_all(e, o * pitch + r.first * inner, out, r.second * inner);
      out += r.second * inner;
    }
  return v;
}

}  // namespace pack
}  // namespace spc
