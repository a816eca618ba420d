// SafeTensors header parsing (host).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace myos {

struct StTensor {
  std::string name;
  std::string dtype;  // header tag, e.g. "BF16"
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;  // byte offsets into the data section
};

// Parses and validates a whole SafeTensors buffer the way the safetensors
// crate's SafeTensors::deserialize does: 8-byte little-endian header length,
// a JSON object header (optional "__metadata__" of strings), data_offsets
// that tile the data section exactly, and byte lengths that match
// shape x dtype size. Returns 0 on success, 1 for a malformed buffer.
// data_offset receives the start of the data section.
int st_parse(const uint8_t* buf, size_t len, std::vector<StTensor>* out, size_t* data_offset,
             std::string* why);

// Element size of a SafeTensors dtype tag; 0 for an unknown tag.
size_t st_dtype_size(const std::string& tag);

}  // namespace myos
