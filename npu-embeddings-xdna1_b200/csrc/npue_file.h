// Host-side reader of the `.npue` weight container: mmap, header checks, the
// JSON directory, and typed access to each tensor's bytes.
//
// The format is the reference's (writer tools/lib/npue.py:261, :790-872;
// reader runtime/src/model.cpp:214-380): a 64-byte little-endian header
// "<4sIII QQQQ 16s" (magic "NPUE", version 1, arch, flags, json_offset,
// json_length, data_offset, data_length), a UTF-8 JSON directory
// {"config": {...}, "tensors": [{name, role, dtype, logical_shape,
// padded_shape, offset, nbytes}, ...]}, and 4096-aligned tensor data.  The
// reader is this library's own; it refuses what the reference refuses (bad
// magic, version, alignment, size mismatch) with the reason.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace nebw {

// A minimal JSON value: enough for the container directory.
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;       // String, and the raw text of a Number
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json *find(const std::string &key) const;
  static Json parse(const std::string &text);  // throws std::runtime_error
};

struct NpueTensor {
  std::string name, role, dtype;
  std::string layout_hash;  // sha256 of the layout descriptor; empty when the entry has none
  // the entry's layout descriptor (kind empty when it has none): a block
  // panel's tile and sub-tile sizes, axis order and element type
  std::string layout_kind, layout_order, layout_inner, layout_dtype;
  int64_t tile_k = 0, tile_n = 0, mac_s = 0, mac_t = 0;
  std::vector<int64_t> padded_shape;
  std::vector<int64_t> shape;
  uint64_t offset = 0, nbytes = 0;
  const uint8_t *data = nullptr;
};

class NpueFile {
 public:
  explicit NpueFile(const std::string &path);  // throws std::runtime_error
  ~NpueFile();
  NpueFile(const NpueFile &) = delete;
  NpueFile &operator=(const NpueFile &) = delete;

  const NpueTensor &tensor(const std::string &name) const;  // throws if absent
  bool has(const std::string &name) const { return tensors_.count(name) != 0; }
  // config values, as the reference reads them (model.cpp:366-380)
  int64_t config_int(const std::string &key) const;
  double config_double(const std::string &key) const;
  std::string config_string(const std::string &key) const;
  bool has_config(const std::string &key) const { return config_.find(key) != nullptr; }
  uint32_t arch() const { return arch_; }

 private:
  std::string path_;
  const uint8_t *base_ = nullptr;
  size_t size_ = 0;
  uint32_t arch_ = 0;
  Json config_;
  std::map<std::string, NpueTensor> tensors_;
};

}  // namespace nebw
