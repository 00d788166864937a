// Two-tier memory allocator for torch's CUDAPluggableAllocator / MemPool.
//
// Reference: mem/custom_allocator.cpp (a CPU allocator with a DDR and an HBM
// tier, sharded free lists, MAX_DDR_MEMORY / MAX_HBM_MEMORY caps and a
// thread-local "allocate on HBM" switch).  On a B200 node the two tiers are
//   device  : GPU HBM3e, stream-ordered cudaMallocAsync / cudaFreeAsync;
//   host    : page-locked, device-mapped host memory (cudaHostAlloc), cached
//             in size classes.  Kernels read and write it in place over the
//             host link (a "DDR" tensor that still lives on the cuda device).
// Each tier honours a byte cap (HARP_MAX_HBM_MEMORY / HARP_MAX_DDR_MEMORY,
// also read as MAX_HBM_MEMORY / MAX_DDR_MEMORY; 0 = unlimited).  A request
// over the cap first releases cached host blocks and then fails (nullptr), which
// torch reports as an out-of-memory error; the reference blocked instead.
//
// Host blocks freed while kernels may still use them carry a CUDA event
// recorded on the freeing stream; a cached block is reused only after its
// event has completed, so no kernel reads memory that was handed out again.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace {

int64_t env_bytes(const char* a, const char* b) {
  const char* v = std::getenv(a);
  if (!v) v = std::getenv(b);
  if (!v) return 0;
  return std::atoll(v);
}

struct Stats {
  std::atomic<int64_t> in_use{0}, cached{0}, peak{0}, allocs{0}, fails{0};
  void add_use(int64_t n) {
    int64_t now = in_use.fetch_add(n) + n;
    int64_t p = peak.load();
    while (now > p && !peak.compare_exchange_weak(p, now)) {
    }
  }
};

// ---------------------------------------------------------------------------
// host tier
// ---------------------------------------------------------------------------
struct HostBlock {
  void* ptr;
  size_t size;
  cudaEvent_t ready;  // completes when the last user stream is done with the block
};

struct HostPool {
  std::mutex mu;
  std::map<size_t, std::vector<HostBlock>> free_;  // size class -> cached blocks
  std::unordered_map<void*, size_t> live_;         // ptr -> size class
  Stats st;
  // read by allocating threads, changed at run time by harp_alloc_set_cap
  std::atomic<int64_t> cap{env_bytes("HARP_MAX_DDR_MEMORY", "MAX_DDR_MEMORY")};

  static size_t size_class(size_t n) {
    if (n <= 512) return 512;
    if (n < (1u << 20)) {
      size_t c = 1024;
      while (c < n) c <<= 1;
      return c;
    }
    const size_t g = 2u << 20;  // 2 MiB granules above 1 MiB
    return (n + g - 1) / g * g;
  }

  void release_cached_locked() {
    for (auto& kv : free_)
      for (auto& b : kv.second) {
        if (b.ready) {
          cudaEventSynchronize(b.ready);
          cudaEventDestroy(b.ready);
        }
        cudaFreeHost(b.ptr);
        st.cached -= (int64_t)b.size;
      }
    free_.clear();
  }

  void* alloc(size_t n) {
    size_t c = size_class(n);
    std::lock_guard<std::mutex> g(mu);
    auto it = free_.find(c);
    if (it != free_.end()) {
      auto& v = it->second;
      for (size_t i = 0; i < v.size(); ++i) {
        if (v[i].ready && cudaEventQuery(v[i].ready) != cudaSuccess) continue;
        HostBlock b = v[i];
        v.erase(v.begin() + (long)i);
        if (b.ready) cudaEventDestroy(b.ready);
        st.cached -= (int64_t)c;
        live_[b.ptr] = c;
        st.add_use((int64_t)c);
        st.allocs++;
        return b.ptr;
      }
    }
    const int64_t limit = cap.load();
    if (limit > 0 && st.in_use.load() + st.cached.load() + (int64_t)c > limit) release_cached_locked();
    if (limit > 0 && st.in_use.load() + (int64_t)c > limit) {
      st.fails++;
      return nullptr;
    }
    void* p = nullptr;
    if (cudaHostAlloc(&p, c, cudaHostAllocPortable | cudaHostAllocMapped) != cudaSuccess) {
      cudaGetLastError();
      release_cached_locked();
      if (cudaHostAlloc(&p, c, cudaHostAllocPortable | cudaHostAllocMapped) != cudaSuccess) {
        cudaGetLastError();
        st.fails++;
        return nullptr;
      }
    }
    live_[p] = c;
    st.add_use((int64_t)c);
    st.allocs++;
    return p;
  }

  void free(void* p, cudaStream_t stream) {
    if (!p) return;
    std::lock_guard<std::mutex> g(mu);
    auto it = live_.find(p);
    if (it == live_.end()) return;
    size_t c = it->second;
    live_.erase(it);
    HostBlock b{p, c, nullptr};
    if (cudaEventCreateWithFlags(&b.ready, cudaEventDisableTiming) == cudaSuccess) {
      if (cudaEventRecord(b.ready, stream) != cudaSuccess) {
        cudaGetLastError();
        cudaEventDestroy(b.ready);
        b.ready = nullptr;
        cudaStreamSynchronize(stream);
      }
    } else {
      cudaGetLastError();
      cudaStreamSynchronize(stream);
    }
    free_[c].push_back(b);
    st.in_use -= (int64_t)c;
    st.cached += (int64_t)c;
  }
};

// ---------------------------------------------------------------------------
// device tier
// ---------------------------------------------------------------------------
struct DevicePool {
  std::mutex mu;
  std::unordered_map<void*, size_t> live_;
  Stats st;
  std::atomic<int64_t> cap{env_bytes("HARP_MAX_HBM_MEMORY", "MAX_HBM_MEMORY")};

  void* alloc(size_t n, int device, cudaStream_t stream) {
    size_t c = (n + 511) / 512 * 512;
    const int64_t limit = cap.load();
    if (limit > 0 && st.in_use.load() + (int64_t)c > limit) {
      st.fails++;
      return nullptr;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    void* p = nullptr;
    cudaError_t e = cudaMallocAsync(&p, c, stream);
    if (prev != device && prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
      cudaGetLastError();
      st.fails++;
      return nullptr;
    }
    std::lock_guard<std::mutex> g(mu);
    live_[p] = c;
    st.add_use((int64_t)c);
    st.allocs++;
    return p;
  }

  void free(void* p, cudaStream_t stream) {
    if (!p) return;
    size_t c = 0;
    {
      std::lock_guard<std::mutex> g(mu);
      auto it = live_.find(p);
      if (it == live_.end()) return;
      c = it->second;
      live_.erase(it);
    }
    cudaFreeAsync(p, stream);
    st.in_use -= (int64_t)c;
  }
};

HostPool& host_pool() {
  static HostPool* p = new HostPool();  // leaked on purpose: frees may arrive during interpreter exit
  return *p;
}
DevicePool& device_pool() {
  static DevicePool* p = new DevicePool();
  return *p;
}

void fill(const Stats& s, long long* out) {
  out[0] = s.in_use.load();
  out[1] = s.cached.load();
  out[2] = s.peak.load();
  out[3] = s.allocs.load();
  out[4] = s.fails.load();
}

}  // namespace

// Entry points with the signatures torch.cuda.memory.CUDAPluggableAllocator expects.
extern "C" {

void* harp_host_malloc(ssize_t size, int device, cudaStream_t stream) {
  (void)device;
  (void)stream;
  return host_pool().alloc((size_t)size);
}

void harp_host_free(void* ptr, ssize_t size, int device, cudaStream_t stream) {
  (void)size;
  (void)device;
  host_pool().free(ptr, stream);
}

void* harp_dev_malloc(ssize_t size, int device, cudaStream_t stream) {
  return device_pool().alloc((size_t)size, device, stream);
}

void harp_dev_free(void* ptr, ssize_t size, int device, cudaStream_t stream) {
  (void)size;
  (void)device;
  device_pool().free(ptr, stream);
}

// tier 0 = host, 1 = device; out = {in_use, cached, peak, allocations, failures}
void harp_alloc_stats(int tier, long long* out) { fill(tier == 0 ? host_pool().st : device_pool().st, out); }

// Drop cached host blocks (waits for their last users).
void harp_host_empty_cache() {
  std::lock_guard<std::mutex> g(host_pool().mu);
  host_pool().release_cached_locked();
}

// Caps can be changed at run time (bytes; 0 = unlimited).
void harp_alloc_set_cap(int tier, long long bytes) {
  if (tier == 0)
    host_pool().cap.store(bytes);
  else
    device_pool().cap.store(bytes);
}
}
