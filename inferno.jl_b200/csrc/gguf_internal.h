// Parsed GGUF file (gguf.cu): the read-only mapping plus its metadata and
// tensor table.  Shared with the engine's loader (engine.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

struct GgufValue {
  uint32_t type = 0;              // GGUF value type
  int64_t i = 0;                  // integer / bool value (uint64 stored bit-for-bit)
  double f = 0.0;                 // float value (integers converted)
  bool is_float = false, is_string = false, u64 = false;
  std::string s;
  uint32_t arr_type = 0;          // arrays: element type, length, first element in the mapping
  uint64_t arr_len = 0;
  const uint8_t* arr_data = nullptr;
};

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  int type = -1;
  uint64_t offset = 0;            // from the start of the data section
  uint64_t nbytes = 0;            // 0 when the type's block size is unknown
};

struct InfernoGguf {
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32, data_offset = 0;
  std::map<std::string, GgufValue> kv;
  std::vector<std::string> kv_order;
  std::vector<GgufTensor> tensors;
};

namespace inf {
int gguf_parse(const uint8_t* p, size_t n, InfernoGguf* g);
}
