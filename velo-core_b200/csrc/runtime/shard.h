// shard.h -- host-side tensor-parallel weight sharding (shard.cpp).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "velo_cuda.h"

namespace velo {

int32_t shard_strategy(const char* name);
int32_t shard_weight(const velo_weight_desc& w, int32_t strategy, int tp, int rank,
                     std::vector<uint8_t>& out, uint64_t& rows_out, uint64_t& cols_out);

}  // namespace velo
