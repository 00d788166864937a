// Host stress test of the two-tier allocator (harp_b200/csrc/alloc.cpp) built
// against tests/native/fake_cuda: eight threads allocate, touch, and free
// blocks of both tiers while other threads change the caps, read the
// statistics and empty the host cache; then a single-thread check that a
// freed host block is not handed out again before its event completes.
// Exit status 0 = every check passed; the sanitizers report races / misuse.
#include <cuda_runtime.h>

#include <sys/types.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

std::atomic<int> g_fake_event_delay{2};

extern "C" {
void* harp_host_malloc(ssize_t size, int device, cudaStream_t stream);
void harp_host_free(void* ptr, ssize_t size, int device, cudaStream_t stream);
void* harp_dev_malloc(ssize_t size, int device, cudaStream_t stream);
void harp_dev_free(void* ptr, ssize_t size, int device, cudaStream_t stream);
void harp_alloc_stats(int tier, long long* out);
void harp_host_empty_cache();
void harp_alloc_set_cap(int tier, long long bytes);
}

namespace {

struct Live {
  void* p;
  size_t n;
  int tier;
  unsigned char tag;
};

int failures = 0;

void check(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

void worker(int id, int iters) {
  std::mt19937 rng(1234 + id);
  FakeStream stream{id};
  std::vector<Live> live;
  for (int it = 0; it < iters; ++it) {
    if (live.size() < 16 && (rng() % 3 != 0 || live.empty())) {
      const int tier = (int)(rng() % 2);
      const size_t n = 1 + rng() % (tier == 0 ? (3u << 20) : 65536u);
      void* p = tier == 0 ? harp_host_malloc((ssize_t)n, 0, &stream) : harp_dev_malloc((ssize_t)n, 0, &stream);
      if (p == nullptr) continue;  // over a cap another thread set
      const unsigned char tag = (unsigned char)(id * 16 + it);
      std::memset(p, tag, n);
      live.push_back({p, n, tier, tag});
    } else {
      const size_t i = rng() % live.size();
      Live b = live[i];
      live.erase(live.begin() + (long)i);
      const unsigned char* c = static_cast<const unsigned char*>(b.p);
      // nobody else wrote into a block this thread still owns
      check(c[0] == b.tag && c[b.n - 1] == b.tag, "block contents intact until freed");
      if (b.tier == 0) harp_host_free(b.p, (ssize_t)b.n, 0, &stream);
      else harp_dev_free(b.p, (ssize_t)b.n, 0, &stream);
    }
  }
  for (const Live& b : live) {
    if (b.tier == 0) harp_host_free(b.p, (ssize_t)b.n, 0, &stream);
    else harp_dev_free(b.p, (ssize_t)b.n, 0, &stream);
  }
}

void meddler(std::atomic<bool>* stop) {
  std::mt19937 rng(99);
  long long st[5];
  while (!stop->load()) {
    switch (rng() % 4) {
      case 0: harp_alloc_set_cap((int)(rng() % 2), (rng() % 2) ? 0 : (long long)(64u << 20)); break;
      case 1: harp_alloc_stats((int)(rng() % 2), st); break;
      case 2: harp_host_empty_cache(); break;
      default: std::this_thread::yield();
    }
  }
  harp_alloc_set_cap(0, 0);
  harp_alloc_set_cap(1, 0);
}

}  // namespace

int main() {
  std::atomic<bool> stop{false};
  std::thread m(meddler, &stop);
  std::vector<std::thread> ws;
  for (int t = 0; t < 8; ++t) ws.emplace_back(worker, t, 4000);
  for (auto& w : ws) w.join();
  stop.store(true);
  m.join();
  long long st[5];
  harp_alloc_stats(0, st);
  check(st[0] == 0, "host tier: nothing in use after every block was freed");
  harp_alloc_stats(1, st);
  check(st[0] == 0, "device tier: nothing in use after every block was freed");

  // a freed host block is reused only once its event reports completion
  harp_host_empty_cache();
  FakeStream s{0};
  g_fake_event_delay.store(2);
  void* a = harp_host_malloc(4096, 0, &s);
  harp_host_free(a, 4096, 0, &s);  // event pending for two more queries
  void* b = harp_host_malloc(4096, 0, &s);
  void* c = harp_host_malloc(4096, 0, &s);
  check(b != a && c != a, "a block whose event is pending is not reused");
  void* d = harp_host_malloc(4096, 0, &s);
  check(d == a, "the block is reused once its event completed");
  for (void* p : {b, c, d}) harp_host_free(p, 4096, 0, &s);
  harp_host_empty_cache();
  harp_alloc_stats(0, st);
  check(st[0] == 0 && st[1] == 0, "host tier empty after empty_cache");

  // caps: an allocation over the cap fails and is counted
  harp_alloc_set_cap(1, 1 << 20);
  harp_alloc_stats(1, st);
  const long long fails0 = st[4];
  void* big = harp_dev_malloc(2 << 20, 0, &s);
  harp_alloc_stats(1, st);
  check(big == nullptr && st[4] == fails0 + 1, "device allocation over the cap fails");
  harp_alloc_set_cap(1, 0);
  std::printf("alloc_stress: %d failures\n", failures);
  return failures == 0 ? 0 : 1;
}
