// Internal interface of the merged-INT8 checkpoint reader (ckpt.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "moe_b200.h"

namespace moe {

struct CkptTensor {
  int dtype = -1;                // MOE_DT_*
  std::vector<int64_t> shape;
  uint64_t bytes = 0;
  int shard = 0;
  uint64_t offset = 0;           // absolute file offset of the payload
};

size_t dtype_bytes(int dt);
const CkptTensor *ckpt_find(const moe_ckpt *c, const std::string &name);
bool ckpt_read(const moe_ckpt *c, const CkptTensor &t, void *dst);

}  // namespace moe
