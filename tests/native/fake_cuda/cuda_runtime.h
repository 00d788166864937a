// Host-only stand-in for the few CUDA runtime calls the harp allocator
// (harp_b200/csrc/alloc.cpp) makes, so that its locking and caching logic can
// run under ThreadSanitizer / AddressSanitizer on a machine without a GPU.
// Memory comes from malloc; an event records a number of queries after which
// it reports completion, which models work still in flight on a stream.
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdlib>

typedef int cudaError_t;
static const cudaError_t cudaSuccess = 0;
static const cudaError_t cudaErrorNotReady = 600;
static const unsigned cudaHostAllocPortable = 1;
static const unsigned cudaHostAllocMapped = 2;
static const unsigned cudaEventDisableTiming = 2;

struct FakeStream {
  int id;
};
typedef FakeStream* cudaStream_t;

struct FakeEvent {
  std::atomic<int> pending{0};
};
typedef FakeEvent* cudaEvent_t;

// queries a freshly recorded event answers "not ready" before it completes
extern std::atomic<int> g_fake_event_delay;

inline cudaError_t cudaHostAlloc(void** p, size_t n, unsigned) {
  *p = std::malloc(n);
  return *p ? cudaSuccess : 2;
}
inline cudaError_t cudaFreeHost(void* p) {
  std::free(p);
  return cudaSuccess;
}
inline cudaError_t cudaMallocAsync(void** p, size_t n, cudaStream_t) {
  *p = std::malloc(n);
  return *p ? cudaSuccess : 2;
}
inline cudaError_t cudaFreeAsync(void* p, cudaStream_t) {
  std::free(p);
  return cudaSuccess;
}
inline cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned) {
  *e = new FakeEvent();
  return cudaSuccess;
}
inline cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) {
  e->pending.store(g_fake_event_delay.load());
  return cudaSuccess;
}
inline cudaError_t cudaEventQuery(cudaEvent_t e) {
  int p = e->pending.load();
  while (p > 0 && !e->pending.compare_exchange_weak(p, p - 1)) {
  }
  return p > 0 ? cudaErrorNotReady : cudaSuccess;
}
inline cudaError_t cudaEventSynchronize(cudaEvent_t e) {
  e->pending.store(0);
  return cudaSuccess;
}
inline cudaError_t cudaEventDestroy(cudaEvent_t e) {
  delete e;
  return cudaSuccess;
}
inline cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
inline cudaError_t cudaGetLastError() { return cudaSuccess; }
inline cudaError_t cudaGetDevice(int* d) {
  *d = 0;
  return cudaSuccess;
}
inline cudaError_t cudaSetDevice(int) { return cudaSuccess; }
