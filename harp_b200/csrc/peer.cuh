// Peer address tables for kernels that read or write other GPUs' memory
// through CUDA IPC mappings (NVLink), shared by comm.cu and ulysses.cu.
#pragma once
#include <ATen/ATen.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "gemm_sm100.h"

namespace harp {
namespace comm {

constexpr int kMaxPeers = 8;

struct PeerTable {
  uint64_t base[kMaxPeers];  // segment base address of each rank (own included)
};

inline PeerTable make_table(const std::vector<int64_t>& ptrs, long long offset) {
  TORCH_CHECK(ptrs.size() <= (size_t)kMaxPeers, "harp_comm: at most ", kMaxPeers, " ranks per group");
  PeerTable t;
  for (int i = 0; i < kMaxPeers; ++i) t.base[i] = 0;
  for (size_t i = 0; i < ptrs.size(); ++i) t.base[i] = (uint64_t)ptrs[i] + offset;
  return t;
}

inline int grid_for(long long work, int threads) {
  const long long want = (work + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(want, (long long)num_sms() * 4));
}

}  // namespace comm
}  // namespace harp
