// Zero-copy safetensors reader (host side, C++).
//
// File layout: an 8-byte little-endian header length N, N bytes of JSON
// ({"name": {"dtype": "BF16", "shape": [..], "data_offsets": [begin, end]}, ...,
// "__metadata__": {"k": "v"}}), then the data section; offsets are relative to
// the start of the data section.  The file is mmapped read-only and tensors are
// returned as views into the mapping.  Every inconsistency (offsets outside the
// file, size != prod(shape) * itemsize, overlapping or unknown dtypes) is an
// error: the reader refuses the file instead of guessing.
//
// Behavioural counterpart of the reference's Checkpoint / TensorView
// (engines/glm5-moe-nvfp4-2b/src/safetensors.h:25-83, safetensors.cc:261); the
// JSON parser and the mapping code here are this build's own.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace rkt_rt {

struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets into the data section
};

// Bytes per element of a safetensors dtype name; 0 if unknown.
int dtype_itemsize(const std::string& dtype);

class SafetensorsFile {
 public:
  explicit SafetensorsFile(const std::string& path);
  ~SafetensorsFile();
  SafetensorsFile(const SafetensorsFile&) = delete;
  SafetensorsFile& operator=(const SafetensorsFile&) = delete;

  const std::string& path() const { return path_; }
  std::vector<std::string> keys() const;
  const TensorInfo& info(const std::string& name) const;
  const std::map<std::string, std::string>& metadata() const { return meta_; }
  // Pointer to the tensor's bytes inside the mapping (valid while this object lives).
  const uint8_t* data(const std::string& name) const;
  uint64_t file_size() const { return size_; }

 private:
  std::string path_;
  int fd_ = -1;
  uint8_t* map_ = nullptr;
  uint64_t size_ = 0;
  uint64_t data_off_ = 0;
  std::map<std::string, TensorInfo> tensors_;
  std::map<std::string, std::string> meta_;
};

}  // namespace rkt_rt
