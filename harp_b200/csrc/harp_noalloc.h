// Public C interface of the allocation-free entry point of the harp_b200
// library.  It has no counterpart in the reference (wxyww2049/HARP has no GPU
// code at all); it exists for callers that cannot call cudaMalloc while they
// run:
//   * a plugin or callback inside another runtime (an inference engine, a
//     graph executor) that plans every byte of device memory ahead of time and
//     forbids allocation during execution;
//   * a process whose device memory is fully reserved by a pool or caching
//     allocator, where cudaMalloc would fail;
//   * a latency-critical loop that cannot afford cudaMalloc/cudaFree, which may
//     synchronize the whole device.
//
// Load the library (harp_b200/_build/harp_b200_C.so) with dlopen or ctypes
// and call the symbol below; the definition is in noalloc_rmsnorm.cu, which
// includes this header so that the compiler checks that both agree.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of harp_rmsnorm_backward_noalloc.
enum HarpNoallocStatus {
  HARP_NOALLOC_OK = 0,
  HARP_NOALLOC_BAD_ARGS = -1,      // null pointer, dim % 8 != 0, rows < 0 or a pointer not 16-byte aligned
  HARP_NOALLOC_TOO_LARGE = -2,     // rows exceed the static scratch (see the size limit below); nothing enqueued
  HARP_NOALLOC_SETUP_FAILED = -3,  // cudaGetDevice or cudaGetSymbolAddress failed
  HARP_NOALLOC_LAUNCH_FAILED = -4, // a kernel launch or the memset of an empty batch failed
};

// Maximum scratch: 2^20 fp32 partial sums (4 MiB, a static __device__ array
// that every GPU which loads the library holds until the process exits).
#define HARP_NOALLOC_SCRATCH_FLOATS (1ll << 20)
// Rows one block may fold into one partial sum (their statistics live in
// 16 KiB of shared memory).
#define HARP_NOALLOC_MAX_ROWS_PER_BLOCK 4096

// RMSNorm backward without any allocation.
//   input, grad_out, grad_input: bf16 [rows, dim] row-major;
//   weight, grad_weight: bf16 [dim];
//   rms: fp32 [rows], the per-row root mean square (not its inverse) that the
//        library's RMSNorm forward (async_op::rmsnorm_forward_out) saves.
//   dim % 8 == 0; input, grad_out, weight and grad_input 16-byte aligned
//   (with rows == 0 the row buffers are not read and may be null).
// Computes grad_input = rstd * (g*w - xhat * mean(g*w*xhat)) and
// grad_weight = sum over rows of g*xhat (rstd = 1/rms, xhat = x*rstd), fp32
// inside, enqueued on `stream` (a cudaStream_t; 0 = the legacy default stream).
// Returns without waiting for the GPU.
//
// Size limit: rows <= HARP_NOALLOC_MAX_ROWS_PER_BLOCK *
//                     floor(HARP_NOALLOC_SCRATCH_FLOATS / dim);
// larger calls return HARP_NOALLOC_TOO_LARGE and enqueue nothing.
//
// Set-up: the first call on each device (with that device current) looks up
// the device address of the scratch array once and caches it for the life of
// the process; make that first call before any stream capture.  The cached
// address is not refreshed after cudaDeviceReset, so the library must not be
// used across a device reset.
//
// Every call shares the one scratch array, which keeps the last call's
// contents.  Each call writes every partial sum it later reads, so nothing
// needs to start at zero; calls that overlap on the GPU (two streams, two
// threads) race on the scratch, so the caller must order them.
int harp_rmsnorm_backward_noalloc(const void* input, const void* grad_out, const void* weight, const float* rms,
                                  void* grad_input, void* grad_weight, long long rows, long long dim, void* stream);

#ifdef __cplusplus
}
#endif
