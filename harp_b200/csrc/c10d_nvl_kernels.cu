// Kernels of the "harp_nvl" torch.distributed backend (c10d_nvl.cpp): NVLink
// peer-memory collectives over a symmetric heap.  Every rank's heap is mapped
// into every peer through CUDA IPC; a rank publishes its heap contents for
// epoch e by storing e into its slot of every peer's flag array (release,
// system scope), and readers wait (acquire, bounded by a timeout that writes
// the error word and returns) before pulling with 16-byte loads.
#include "c10d_nvl_kernels.h"
#include "common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace harp {
namespace nvl {
namespace {

__global__ void signal_k(Peers flags, int world, int slot, unsigned value) {
  const int r = threadIdx.x;
  if (r >= world) return;
  __threadfence_system();
  st_release_sys(reinterpret_cast<unsigned*>(flags.base[r]) + slot, value);
}

__global__ void wait_k(const unsigned* flags, int first, int count, unsigned value, unsigned long long timeout_ns,
                       int* err) {
  const int i = threadIdx.x;
  if (i < count) wait_flag_geq(flags + first + i, value, timeout_ns, err, 300 + i);
}

__device__ __forceinline__ bool wait_sources(const unsigned* flags, int slot, int world, int only, unsigned value,
                                             unsigned long long timeout_ns, int* err) {
  if (threadIdx.x < world && (only < 0 || (int)threadIdx.x == only))
    wait_flag_geq(flags + slot + threadIdx.x, value, timeout_ns, err, 310 + threadIdx.x);
  __syncthreads();
  return *(volatile int*)err == 0;
}

// dst[r * bytes + i] = heap_r[off + i], each source after its flag (or only
// source `only` when >= 0, landing at dst directly).  bytes % 16 == 0.
__global__ void gather_k(Peers heap, long long off, long long bytes, char* dst, int world, int rank, int only,
                         const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err) {
  if (!wait_sources(flags, slot, world, only, value, timeout_ns, err)) return;
  const long long vecs = bytes / 16;
  for (int step = 0; step < world; ++step) {
    const int r = only >= 0 ? only : (rank + step) % world;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(heap.base[r]) + off);
    uint4* d = reinterpret_cast<uint4*>(dst + (only >= 0 ? 0 : (long long)r * bytes));
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < vecs;
         v += (long long)gridDim.x * blockDim.x)
      d[v] = src[v];
    if (only >= 0) break;
  }
}

// dst[r * blk + i] = heap_r[rank * blk + i]: block `rank` of every peer's buffer.
__global__ void alltoall_k(Peers heap, long long blk, char* dst, int world, int rank, const unsigned* flags, int slot,
                           unsigned value, unsigned long long timeout_ns, int* err) {
  if (!wait_sources(flags, slot, world, -1, value, timeout_ns, err)) return;
  const long long vecs = blk / 16;
  for (int step = 0; step < world; ++step) {
    const int r = (rank + step) % world;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(heap.base[r]) + (long long)rank * blk);
    uint4* d = reinterpret_cast<uint4*>(dst + (long long)r * blk);
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < vecs;
         v += (long long)gridDim.x * blockDim.x)
      d[v] = src[v];
  }
}

template <typename T>
struct Acc {
  using type = float;
};
template <>
struct Acc<double> {
  using type = double;
};
template <>
struct Acc<int> {
  using type = long long;
};
template <>
struct Acc<long long> {
  using type = long long;
};

template <typename T>
__device__ __forceinline__ typename Acc<T>::type to_acc(T x) {
  return (typename Acc<T>::type)x;
}
template <>
__device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_acc<__half>(__half x) {
  return __half2float(x);
}
template <typename T, typename A>
__device__ __forceinline__ T from_acc(A x) {
  return (T)x;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16, float>(float x) {
  return __float2bfloat16(x);
}
template <>
__device__ __forceinline__ __half from_acc<__half, float>(float x) {
  return __float2half(x);
}

// dst[i] = op over ranks r (fixed order 0..world-1) of heap_r[src_off + i]
template <typename T>
__global__ void reduce_k(Peers heap, long long src_off, long long count, T* dst, int world, int op,
                         const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err) {
  if (!wait_sources(flags, slot, world, -1, value, timeout_ns, err)) return;
  using A = typename Acc<T>::type;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x) {
    A acc = to_acc<T>(reinterpret_cast<const T*>(heap.base[0])[src_off + i]);
    for (int r = 1; r < world; ++r) {
      const A x = to_acc<T>(reinterpret_cast<const T*>(heap.base[r])[src_off + i]);
      switch (op) {
        case kMax: acc = x > acc ? x : acc; break;
        case kMin: acc = x < acc ? x : acc; break;
        case kProduct: acc = acc * x; break;
        default: acc = acc + x; break;
      }
    }
    if (op == kAvg) acc = acc / (A)world;
    dst[i] = from_acc<T, A>(acc);
  }
}

int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > 148 * 4) g = 148 * 4;
  return (int)g;
}

}  // namespace

void launch_signal(Peers flags, int world, int slot, unsigned value, cudaStream_t s) {
  signal_k<<<1, 32, 0, s>>>(flags, world, slot, value);
}

void launch_wait(const unsigned* flags, int first, int count, unsigned value, unsigned long long timeout_ns,
                 int* err, cudaStream_t s) {
  wait_k<<<1, 32, 0, s>>>(flags, first, count, value, timeout_ns, err);
}

void launch_gather(Peers heap, long long off, long long bytes, void* dst, int world, int rank, int only,
                   const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err,
                   cudaStream_t s) {
  gather_k<<<grid_for(bytes / 16, 512), 512, 0, s>>>(heap, off, bytes, reinterpret_cast<char*>(dst), world, rank,
                                                     only, flags, slot, value, timeout_ns, err);
}

void launch_alltoall(Peers heap, long long blk, void* dst, int world, int rank, const unsigned* flags, int slot,
                     unsigned value, unsigned long long timeout_ns, int* err, cudaStream_t s) {
  alltoall_k<<<grid_for(blk / 16, 512), 512, 0, s>>>(heap, blk, reinterpret_cast<char*>(dst), world, rank, flags, slot,
                                                     value, timeout_ns, err);
}

bool launch_reduce(DType dt, Peers heap, long long src_off, long long count, void* dst, int world, int op,
                   const unsigned* flags, int slot, unsigned value, unsigned long long timeout_ns, int* err,
                   cudaStream_t s) {
  const int threads = 512, grid = grid_for(count, threads);
  switch (dt) {
    case DType::kF32:
      reduce_k<float><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<float*>(dst), world, op, flags,
                                               slot, value, timeout_ns, err);
      return true;
    case DType::kF64:
      reduce_k<double><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<double*>(dst), world, op, flags,
                                                slot, value, timeout_ns, err);
      return true;
    case DType::kBF16:
      reduce_k<__nv_bfloat16><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<__nv_bfloat16*>(dst),
                                                       world, op, flags, slot, value, timeout_ns, err);
      return true;
    case DType::kF16:
      reduce_k<__half><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<__half*>(dst), world, op, flags,
                                                slot, value, timeout_ns, err);
      return true;
    case DType::kI32:
      reduce_k<int><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<int*>(dst), world, op, flags, slot,
                                             value, timeout_ns, err);
      return true;
    case DType::kI64:
      reduce_k<long long><<<grid, threads, 0, s>>>(heap, src_off, count, reinterpret_cast<long long*>(dst), world, op,
                                                   flags, slot, value, timeout_ns, err);
      return true;
  }
  return false;
}

}  // namespace nvl
}  // namespace harp
