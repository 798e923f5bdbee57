// GGUF v3 reader for the host side of the library, following go-semantica's
// internal/gguf (reader.go:98-178, format.go) and parseConfig
// (internal/runtime/model.go:424-517). The Go host keeps its own loader and
// passes tensor views to sem_model_load; this reader serves callers without
// one (and the tests).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "../../../include/semantica_b200.h"

namespace sem {

struct GgufTensor {
  std::string name;
  uint32_t dtype = 0;
  std::vector<uint64_t> dims;
  uint64_t offset = 0;  // relative to the data section
  uint64_t size = 0;    // bytes (format.go BlockSize rule)
};

struct GgufFile {
  const uint8_t* data = nullptr;  // mmap'd file
  size_t len = 0;
  size_t data_off = 0;            // start of tensor data, 32-byte aligned (reader.go:175)
  std::map<std::string, uint32_t> u32;
  std::map<std::string, float> f32;
  std::map<std::string, std::string> str;
  std::map<std::string, uint64_t> array_len;
  std::vector<GgufTensor> tensors;

  ~GgufFile();
  // Returns SEM_OK or an error code with the message set.
  int open(const char* path);
  const GgufTensor* find(const std::string& name) const;
  const uint8_t* tensor_data(const GgufTensor& t) const { return data + data_off + t.offset; }

 private:
  void* map_ = nullptr;
  size_t map_len_ = 0;
};

// parseConfig (model.go:424-517).
int gguf_config(const GgufFile& f, sem_model_config* cfg);

}  // namespace sem
