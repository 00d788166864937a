// Host interface of the harp_nvl collective kernels (c10d_nvl_kernels.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace harp {
namespace nvl {

constexpr int kMaxRanks = 8;
struct Peers {
  uint64_t base[kMaxRanks];
};

enum class DType { kF32, kF64, kBF16, kF16, kI32, kI64 };
enum ReduceOpCode { kSum = 0, kAvg = 1, kMax = 2, kMin = 3, kProduct = 4 };

void launch_signal(Peers flags, int world, int slot, unsigned value, cudaStream_t s);
void launch_wait(const unsigned* flags, int first, int count, unsigned value, unsigned long long timeout_ns,
                 int* err, cudaStream_t s);
void launch_gather(Peers heap, long long off, long long bytes, void* dst, int world, int rank, int only,
                   const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err,
                   cudaStream_t s);
void launch_alltoall(Peers heap, long long blk, void* dst, int world, int rank, const unsigned* flags, int slot,
                     unsigned value, unsigned long long timeout_ns, int* err, cudaStream_t s);
bool launch_reduce(DType dt, Peers heap, long long src_off, long long count, void* dst, int world, int op,
                   const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err,
                   cudaStream_t s);

}  // namespace nvl
}  // namespace harp
