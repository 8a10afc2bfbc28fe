// Checkpoint tensors as the loaders see them (host only; see checkpoint.cu).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/uocr_moe.h"

namespace uocr_b200 {

struct CkTensor {
  int dtype;  // uocr_dtype
  std::vector<int64_t> shape;
  const void* data;  // into the shard's read-only mapping
  uint64_t bytes;
};

// Nullptr when no shard holds the name.
const CkTensor* checkpoint_find(const uocr_checkpoint* ckpt, const std::string& name);
const char* dtype_name(int dtype);

}  // namespace uocr_b200
