// Checkpoint layout: a stage pack is a directory with an index (`stagepack_index.json`)
// and data files holding each tensor as one contiguous region.
//
//   index       format tag, model id, free-form metadata (JSON), and per tensor: name,
//               dtype, shape, bytes per element, data file, offset, bytes, content
//               fingerprint. Written last and atomically (temporary + rename), so a
//               pack directory either has a complete index or none.
//   data files  `data_NNNN.bin`, regions 4 KiB aligned (page- and O_DIRECT-friendly),
//               a new file once one would pass 4 GiB
//   resolve     a tensor spec (name, dtype, shape, bytes per element) -> its region
//               (file path, offset, bytes); fails closed on an unknown name
//               (NotFound) or any dtype / rank / shape / size disagreement
//               (SchemaError) — never returns a region of the wrong shape
//   read        whole tensor; a leading-dimension row range (an expert-parallel
//               rank's experts: one contiguous range); or a tensor-parallel shard
//               computed by the TP shard engine (tp_shard.h): a split on the leading
//               dimension is one contiguous range per part, a split on an inner
//               dimension gathers one chunk per outer row at the full row pitch, and
//               the destination must be exactly the shard's bytes
//
// Reference behaviour: the stage-pack resolve contract and the shard read
// (crates/spark-abi/vendor/sparkpipe/model-families/glm52/include/sparkpipe/
// spark_glm52_stagepack.h:11-52, include/sparkpipe/spark_tp_shard.h:132-148). The
// reference ships declarations only; the file format here is this framework's own.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"
#include "tp_shard.h"

namespace spc {
namespace pack {

constexpr const char* kIndexFile = "stagepack_index.json";
constexpr const char* kFormat = "sparkpipe_b200.stagepack.v1";
constexpr uint32_t kMaxRank = 8;
constexpr uint64_t kAlign = 4096;
constexpr uint64_t kFileLimit = 4ull << 30;
constexpr size_t kPathBytes = 4096;

struct Entry {
  std::string name, dtype, file;
  std::vector<uint64_t> shape;
  uint64_t bytes_per_element = 0, offset = 0, bytes = 0, fingerprint = 0;
};

struct Region {
  std::string file_path;
  uint64_t file_offset = 0, tensor_bytes = 0;
};

// 64-bit content fingerprint (four multiply-rotate lanes over 32-byte blocks): fast
// enough to check GB-sized tensors at load, not a cryptographic hash.
uint64_t fingerprint(const void* data, size_t n);

class Writer {
 public:
  Writer(const std::string& root, const std::string& model_id, const std::string& metadata_json);
  ~Writer();
  void add(const std::string& name, const std::string& dtype, const std::vector<uint64_t>& shape,
           uint64_t bytes_per_element, const void* data, uint64_t bytes);
  void finish();  // writes the index; no add after it
  uint64_t bytes_written() const { return total_; }

 private:
  void open_next();
  std::string root_, model_id_, metadata_;
  std::vector<Entry> entries_;
  int fd_ = -1;
  uint32_t file_no_ = 0;
  uint64_t pos_ = 0, total_ = 0;
  bool finished_ = false;
};

class Pack {
 public:
  static Pack open(const std::string& root);
  const std::string& root() const { return root_; }
  const std::string& model_id() const { return model_id_; }
  const std::string& metadata() const { return metadata_; }
  std::vector<std::string> names() const;
  const Entry& entry(const std::string& name) const;  // NotFound
  Region resolve(const std::string& name, const std::string& dtype, const std::vector<uint64_t>& shape,
                 uint64_t bytes_per_element) const;
  void read(const std::string& name, void* dst, uint64_t dst_bytes, bool verify) const;
  // rows [row0, row0 + rows) of the leading dimension
  void read_rows(const std::string& name, uint64_t row0, uint64_t rows, void* dst, uint64_t dst_bytes) const;
  tp::View read_shard(const std::string& name, const tp::Shape& shape, const tp::Geometry& g, void* dst,
                      uint64_t dst_bytes) const;

 private:
  void pread_all(const Entry& e, uint64_t rel, void* dst, uint64_t n) const;
  std::string root_, model_id_, metadata_;
  std::vector<Entry> entries_;
  std::unordered_map<std::string, size_t> by_name_;
};

}  // namespace pack
}  // namespace spc
