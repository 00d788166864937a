// "harp_nvl": a torch.distributed (c10d) backend for the GPUs of one node that
// runs every collective as harp kernels over NVLink peer memory.
//
// Reference counterpart: the HMPI c10d backend registered for CPU tensors
// (hmpi/ProcessGroupHMPI.cpp:50-76 registration, :579-1234 collectives, a
// worker thread per group).  Here, per group:
//   * a symmetric heap (HARP_NVL_HEAP_MB, default 256 MiB per rank) and a flag
//     array are cudaMalloc'ed on every rank and mapped into every peer with
//     CUDA IPC; the handles travel through the group's c10d Store;
//   * a collective copies its input into the local heap, stores the epoch into
//     its DATA slot of every peer's flags, and a kernel on every rank waits for
//     the peers' DATA flags (bounded: on timeout it writes the error word and
//     returns) and pulls what it needs with 16-byte loads; then the rank
//     stores the epoch into its ACK slot, which the next collective waits for
//     before overwriting the heap;
//   * all of it is issued on the caller's current CUDA stream, so a collective
//     is ordered like any kernel and works inside CUDA graphs; Work objects
//     hold a CUDA event (wait() = stream wait, synchronize() = host wait plus
//     an error-word check that raises).
// Collectives: allreduce (sum / avg / min / max / product; one-shot up to
// 1 MiB, reduce-scatter + all-gather above), broadcast, allgather
// (+ _allgather_base), reduce_scatter (+ _reduce_scatter_base), alltoall_base
// with equal splits, barrier.  Every rank sums in rank order, so all ranks
// get bit-identical results.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/chrono.h>
#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <torch/csrc/distributed/c10d/Types.hpp>
#include <torch/csrc/distributed/c10d/Work.hpp>
#include <torch/extension.h>

#include <cstdlib>
#include <cstring>

#include "c10d_nvl_kernels.h"

namespace harp {
namespace nvl {

constexpr int kData = 0, kAck = kMaxRanks, kData2 = 2 * kMaxRanks, kNumFlags = 3 * kMaxRanks;

int64_t env_int(const char* k, int64_t def) {
  const char* v = std::getenv(k);
  return v ? std::atoll(v) : def;
}

DType dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return DType::kF32;
    case at::kDouble: return DType::kF64;
    case at::kBFloat16: return DType::kBF16;
    case at::kHalf: return DType::kF16;
    case at::kInt: return DType::kI32;
    case at::kLong: return DType::kI64;
    default: TORCH_CHECK(false, "harp_nvl: unsupported dtype ", t.scalar_type());
  }
}

int op_of(const c10d::ReduceOp& op) {
  switch (op.op_) {
    case c10d::ReduceOp::SUM: return kSum;
    case c10d::ReduceOp::AVG: return kAvg;
    case c10d::ReduceOp::MAX: return kMax;
    case c10d::ReduceOp::MIN: return kMin;
    case c10d::ReduceOp::PRODUCT: return kProduct;
    default: TORCH_CHECK(false, "harp_nvl: unsupported reduce op");
  }
}

class NVLWork : public c10d::Work {
 public:
  NVLWork(int rank, c10d::OpType type, std::vector<at::Tensor> outputs, at::Tensor err, cudaStream_t stream)
      : c10d::Work(rank, type), outputs_(std::move(outputs)), err_(std::move(err)) {
    event_.record(at::cuda::getStreamFromExternal(stream, err_.device().index()));
  }
  bool isCompleted() override { return event_.query(); }
  bool isSuccess() const override { return true; }
  bool wait(std::chrono::milliseconds) override {
    event_.block(at::cuda::getCurrentCUDAStream(err_.device().index()));
    return true;
  }
  void synchronize() override {
    event_.synchronize();
    auto e = err_.cpu();
    const int* w = e.data_ptr<int>();
    TORCH_CHECK(w[0] == 0, "harp_nvl: a peer did not answer in time (error ", w[0], " at site ", w[1],
                ", value ", w[2], ")");
  }
  c10::intrusive_ptr<c10::ivalue::Future> getFuture() override {
    synchronize();
    auto fut = c10::make_intrusive<c10::ivalue::Future>(c10::ListType::create(c10::TensorType::get()));
    fut->markCompleted(c10::IValue(outputs_));
    return fut;
  }
  std::vector<at::Tensor> result() override { return outputs_; }

 private:
  std::vector<at::Tensor> outputs_;
  at::Tensor err_;
  at::cuda::CUDAEvent event_;
};

class NVLBackend : public c10d::Backend {
 public:
  NVLBackend(const c10::intrusive_ptr<c10d::Store>& store, int rank, int size, std::chrono::milliseconds timeout)
      : c10d::Backend(rank, size), timeout_(timeout) {
    TORCH_CHECK(size <= kMaxRanks, "harp_nvl: at most ", kMaxRanks, " ranks (one node)");
    device_ = c10::cuda::current_device();
    c10::cuda::CUDAGuard g(device_);
    heap_bytes_ = (size_t)env_int("HARP_NVL_HEAP_MB", 256) << 20;
    const double tsec = env_int("HARP_NVL_TIMEOUT_S", std::max<int64_t>(1, timeout.count() / 1000));
    timeout_ns_ = (unsigned long long)(tsec * 1e9);
    C10_CUDA_CHECK(cudaMalloc(&heap_, heap_bytes_));
    C10_CUDA_CHECK(cudaMalloc(&flags_, kNumFlags * sizeof(unsigned)));
    C10_CUDA_CHECK(cudaMemset(flags_, 0, kNumFlags * sizeof(unsigned)));
    err_ = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device_));
    cudaIpcMemHandle_t hh, hf;
    C10_CUDA_CHECK(cudaIpcGetMemHandle(&hh, heap_));
    C10_CUDA_CHECK(cudaIpcGetMemHandle(&hf, flags_));
    std::vector<uint8_t> mine(2 * sizeof(cudaIpcMemHandle_t));
    std::memcpy(mine.data(), &hh, sizeof(hh));
    std::memcpy(mine.data() + sizeof(hh), &hf, sizeof(hf));
    store->set("harp_nvl/h/" + std::to_string(rank), mine);
    for (int r = 0; r < size; ++r) {
      if (r == rank) {
        heap_peers_.base[r] = (uint64_t)heap_;
        flag_peers_.base[r] = (uint64_t)flags_;
        continue;
      }
      auto v = store->get("harp_nvl/h/" + std::to_string(r));
      TORCH_CHECK(v.size() == mine.size(), "harp_nvl: bad IPC handle from rank ", r);
      cudaIpcMemHandle_t ph, pf;
      std::memcpy(&ph, v.data(), sizeof(ph));
      std::memcpy(&pf, v.data() + sizeof(ph), sizeof(pf));
      void *p1 = nullptr, *p2 = nullptr;
      C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p1, ph, cudaIpcMemLazyEnablePeerAccess));
      C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p2, pf, cudaIpcMemLazyEnablePeerAccess));
      heap_peers_.base[r] = (uint64_t)p1;
      flag_peers_.base[r] = (uint64_t)p2;
      opened_.push_back(p1);
      opened_.push_back(p2);
    }
    for (int r = size; r < kMaxRanks; ++r) heap_peers_.base[r] = flag_peers_.base[r] = 0;
    // everyone mapped everyone before the first collective
    store->set("harp_nvl/ready/" + std::to_string(rank), std::vector<uint8_t>{1});
    std::vector<std::string> keys;
    for (int r = 0; r < size; ++r) keys.push_back("harp_nvl/ready/" + std::to_string(r));
    store->wait(keys);
  }

  ~NVLBackend() override {
    try {
      c10::cuda::CUDAGuard g(device_);
      cudaDeviceSynchronize();
      for (void* p : opened_) cudaIpcCloseMemHandle(p);
      cudaFree(heap_);
      cudaFree(flags_);
    } catch (...) {
    }
  }

  const std::string getBackendName() const override { return "harp_nvl"; }

  c10::intrusive_ptr<c10d::Work> broadcast(std::vector<at::Tensor>& tensors,
                                          const c10d::BroadcastOptions& opts) override {
    auto& t = single(tensors);
    const int root = (int)opts.rootRank;
    cudaStream_t s = stream();
    run_chunks(t.nbytes(), heap_bytes_, [&](size_t off, size_t nb) {
      const unsigned e = begin();
      if (rank_ == root) copy_in(t, off, 0, nb, s);
      signal(kData, e, s);
      if (rank_ != root) {
        char* dst = static_cast<char*>(t.data_ptr()) + off;
        if (nb % 16 == 0)
          launch_gather(heap_peers_, 0, nb, dst, size_, rank_, root, flags_, kData, e, timeout_ns_, err(), s);
        else
          gather_unaligned(0, nb, dst, root, kData, e, s);
      }
      end(e, s);
    }, t);
    return work(c10d::OpType::BROADCAST, {t});
  }

  c10::intrusive_ptr<c10d::Work> allreduce(std::vector<at::Tensor>& tensors,
                                          const c10d::AllreduceOptions& opts) override {
    auto& t = single(tensors);
    const int op = op_of(opts.reduceOp);
    const DType dt = dtype_of(t);
    const size_t esz = t.element_size();
    cudaStream_t s = stream();
    const size_t half = heap_bytes_ / 2;
    // elements per pass: one-shot passes up to 1 MiB, two-phase passes up to half the heap
    const size_t n_all = t.numel();
    size_t done = 0;
    while (done < n_all) {
      const size_t left = n_all - done;
      if (left * esz <= (1u << 20)) {
        const unsigned e = begin();
        copy_in(t, done * esz, 0, left * esz, s);
        signal(kData, e, s);
        launch_reduce(dt, heap_peers_, 0, left, static_cast<char*>(t.data_ptr()) + done * esz, size_, op, flags_,
                      kData, e, timeout_ns_, err(), s);
        end(e, s);
        done = n_all;
        break;
      }
      // two-phase: chunk per rank a multiple of 16 bytes
      const size_t unit = 16 / std::min<size_t>(esz, 16);
      size_t per = std::min(left, half / esz);
      size_t chunk = (per + size_ - 1) / size_;
      chunk = (chunk + unit - 1) / unit * unit;
      per = std::min(left, chunk * size_);
      const unsigned e = begin();
      copy_in(t, done * esz, 0, per * esz, s);
      signal(kData, e, s);
      const size_t lo = std::min(per, chunk * rank_), hi = std::min(per, chunk * (rank_ + 1));
      char* stage2 = static_cast<char*>(heap_) + half;
      if (hi > lo)
        launch_reduce(dt, heap_peers_, lo, hi - lo, stage2, size_, op, flags_, kData, e, timeout_ns_, err(), s);
      else
        launch_wait(flags_, kData, size_, e, timeout_ns_, err(), s);
      signal(kData2, e, s);
      // all-gather the reduced chunks (each rank's chunk sits at heap + half)
      for (int r = 0; r < size_; ++r) {
        const size_t rlo = std::min(per, chunk * r), rhi = std::min(per, chunk * (r + 1));
        if (rhi <= rlo) continue;
        const size_t nb = (rhi - rlo) * esz;
        if (nb % 16 == 0)
          launch_gather(heap_peers_, half, nb, static_cast<char*>(t.data_ptr()) + (done + rlo) * esz, size_, rank_,
                        r, flags_, kData2, e, timeout_ns_, err(), s);
        else
          gather_unaligned(half, nb, static_cast<char*>(t.data_ptr()) + (done + rlo) * esz, r, kData2, e, s);
      }
      end(e, s);
      done += per;
    }
    return work(c10d::OpType::ALLREDUCE, {t});
  }

  c10::intrusive_ptr<c10d::Work> _allgather_base(at::Tensor& out, at::Tensor& in,
                                                const c10d::AllgatherOptions&) override {
    TORCH_CHECK(out.is_contiguous() && in.is_contiguous() && out.numel() == in.numel() * size_,
                "harp_nvl allgather: out = world x in, contiguous");
    cudaStream_t s = stream();
    const size_t nb = in.nbytes();
    run_chunks(nb, heap_bytes_, [&](size_t off, size_t len) {
      const unsigned e = begin();
      copy_in(in, off, 0, len, s);
      signal(kData, e, s);
      for (int r = 0; r < size_; ++r) {
        char* dst = static_cast<char*>(out.data_ptr()) + r * nb + off;
        if (len % 16 == 0)
          launch_gather(heap_peers_, 0, len, dst, size_, rank_, r, flags_, kData, e, timeout_ns_, err(), s);
        else
          gather_unaligned(0, len, dst, r, kData, e, s);
      }
      end(e, s);
    }, in);
    return work(c10d::OpType::_ALLGATHER_BASE, {out});
  }

  c10::intrusive_ptr<c10d::Work> allgather(std::vector<std::vector<at::Tensor>>& outs, std::vector<at::Tensor>& ins,
                                          const c10d::AllgatherOptions& opts) override {
    auto& in = single(ins);
    TORCH_CHECK(outs.size() == 1 && (int)outs[0].size() == size_, "harp_nvl allgather: one list of world tensors");
    auto flat = at::empty({in.numel() * size_}, in.options());
    auto inc = in.contiguous();
    _allgather_base(flat, inc, opts);
    for (int r = 0; r < size_; ++r) outs[0][r].copy_(flat.narrow(0, r * in.numel(), in.numel()).view_as(outs[0][r]));
    return work(c10d::OpType::ALLGATHER, outs[0]);
  }

  c10::intrusive_ptr<c10d::Work> _reduce_scatter_base(at::Tensor& out, at::Tensor& in,
                                                     const c10d::ReduceScatterOptions& opts) override {
    TORCH_CHECK(out.is_contiguous() && in.is_contiguous() && in.numel() == out.numel() * size_,
                "harp_nvl reduce_scatter: in = world x out, contiguous");
    const int op = op_of(opts.reduceOp);
    const size_t esz = in.element_size(), n = out.numel();
    TORCH_CHECK(in.nbytes() <= heap_bytes_, "harp_nvl reduce_scatter: input larger than the heap (",
                heap_bytes_ >> 20, " MiB; set HARP_NVL_HEAP_MB)");
    cudaStream_t s = stream();
    const unsigned e = begin();
    copy_in(in, 0, 0, in.nbytes(), s);
    signal(kData, e, s);
    launch_reduce(dtype_of(in), heap_peers_, (long long)(rank_ * n), (long long)n, out.data_ptr(), size_, op, flags_,
                  kData, e, timeout_ns_, err(), s);
    (void)esz;
    end(e, s);
    return work(c10d::OpType::_REDUCE_SCATTER_BASE, {out});
  }

  c10::intrusive_ptr<c10d::Work> reduce_scatter(std::vector<at::Tensor>& outs,
                                               std::vector<std::vector<at::Tensor>>& ins,
                                               const c10d::ReduceScatterOptions& opts) override {
    auto& out = single(outs);
    TORCH_CHECK(ins.size() == 1 && (int)ins[0].size() == size_, "harp_nvl reduce_scatter: one list of world tensors");
    auto flat = at::cat(ins[0]).contiguous().view({-1});
    auto o = out.is_contiguous() ? out : out.contiguous();
    auto ov = o.view({-1});
    _reduce_scatter_base(ov, flat, opts);
    if (!out.is_contiguous()) out.copy_(o);
    return work(c10d::OpType::REDUCE_SCATTER, {out});
  }

  c10::intrusive_ptr<c10d::Work> alltoall_base(at::Tensor& out, at::Tensor& in, std::vector<int64_t>& out_splits,
                                              std::vector<int64_t>& in_splits,
                                              const c10d::AllToAllOptions&) override {
    TORCH_CHECK(out_splits.empty() && in_splits.empty(), "harp_nvl alltoall: equal splits only");
    TORCH_CHECK(out.is_contiguous() && in.is_contiguous() && out.numel() == in.numel() && in.numel() % size_ == 0,
                "harp_nvl alltoall: contiguous, equal sizes divisible by world");
    const size_t blk = in.nbytes() / size_;
    TORCH_CHECK(blk % 16 == 0, "harp_nvl alltoall: per-rank block must be a multiple of 16 bytes");
    TORCH_CHECK(in.nbytes() <= heap_bytes_, "harp_nvl alltoall: input larger than the heap");
    cudaStream_t s = stream();
    const unsigned e = begin();
    copy_in(in, 0, 0, in.nbytes(), s);
    signal(kData, e, s);
    launch_alltoall(heap_peers_, (long long)blk, out.data_ptr(), size_, rank_, flags_, kData, e, timeout_ns_, err(),
                    s);
    end(e, s);
    return work(c10d::OpType::ALLTOALL_BASE, {out});
  }

  c10::intrusive_ptr<c10d::Work> barrier(const c10d::BarrierOptions&) override {
    cudaStream_t s = stream();
    const unsigned e = begin();
    signal(kData, e, s);
    launch_wait(flags_, kData, size_, e, timeout_ns_, err(), s);
    end(e, s);
    auto w = work(c10d::OpType::BARRIER, {});
    w->synchronize();  // a barrier blocks the host, like the other backends' barrier
    return w;
  }

 private:
  static at::Tensor& single(std::vector<at::Tensor>& ts) {
    TORCH_CHECK(ts.size() == 1, "harp_nvl: one tensor per call");
    TORCH_CHECK(ts[0].is_cuda(), "harp_nvl: CUDA tensors only");
    return ts[0];
  }
  static size_t pad16(size_t n) { return (n + 15) / 16 * 16; }
  cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(device_).stream(); }
  int* err() { return err_.data_ptr<int>(); }

  // next epoch; the heap may be overwritten once every peer acked the previous one
  unsigned begin() {
    const unsigned e = ++epoch_;
    if (e > 1) launch_wait(flags_, kAck, size_, e - 1, timeout_ns_, err(), stream());
    return e;
  }
  void signal(int slot, unsigned e, cudaStream_t s) { launch_signal(flag_peers_, size_, slot + rank_, e, s); }
  void end(unsigned e, cudaStream_t s) { signal(kAck, e, s); }

  void copy_in(const at::Tensor& t, size_t src_off, size_t heap_off, size_t nb, cudaStream_t s) {
    TORCH_CHECK(t.is_contiguous(), "harp_nvl: contiguous tensors only");
    TORCH_CHECK(heap_off + nb <= heap_bytes_, "harp_nvl: heap too small");
    C10_CUDA_CHECK(cudaMemcpyAsync(static_cast<char*>(heap_) + heap_off, static_cast<const char*>(t.data_ptr()) + src_off,
                                   nb, cudaMemcpyDeviceToDevice, s));
  }

  // a source block whose size is not a multiple of 16 bytes: pull the padded
  // block into a scratch tensor, then copy the exact bytes
  void gather_unaligned(size_t heap_off, size_t nb, char* dst, int src, int slot, unsigned e, cudaStream_t s) {
    auto tmp = at::empty({(int64_t)pad16(nb)}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device_));
    launch_gather(heap_peers_, heap_off, pad16(nb), tmp.data_ptr(), size_, rank_, src, flags_, slot, e, timeout_ns_,
                  err(), s);
    C10_CUDA_CHECK(cudaMemcpyAsync(dst, tmp.data_ptr(), nb, cudaMemcpyDeviceToDevice, s));
  }

  template <typename F>
  void run_chunks(size_t total, size_t cap, F&& f, const at::Tensor& t) {
    TORCH_CHECK(t.is_contiguous(), "harp_nvl: contiguous tensors only");
    cap = cap / 16 * 16;
    for (size_t off = 0; off < total; off += cap) f(off, std::min(cap, total - off));
    if (total == 0) return;
  }

  c10::intrusive_ptr<c10d::Work> work(c10d::OpType type, std::vector<at::Tensor> outs) {
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return c10::make_intrusive<NVLWork>(rank_, type, std::move(outs), err_, stream());
  }

  std::chrono::milliseconds timeout_;
  unsigned long long timeout_ns_ = 0;
  c10::DeviceIndex device_ = 0;
  size_t heap_bytes_ = 0;
  void* heap_ = nullptr;
  unsigned* flags_ = nullptr;
  Peers heap_peers_{}, flag_peers_{};
  std::vector<void*> opened_;
  at::Tensor err_;
  unsigned epoch_ = 0;
};

c10::intrusive_ptr<c10d::Backend> create_backend(const c10::intrusive_ptr<c10d::Store>& store, int64_t rank,
                                                 int64_t size, const std::chrono::duration<float>& timeout) {
  return c10::make_intrusive<NVLBackend>(store, (int)rank, (int)size,
                                         std::chrono::duration_cast<std::chrono::milliseconds>(timeout));
}

}  // namespace nvl
}  // namespace harp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "harp_nvl: NVLink peer-memory torch.distributed backend";
  m.def("create_backend", &harp::nvl::create_backend, "create a harp_nvl c10d backend",
        pybind11::arg("store"), pybind11::arg("rank"), pybind11::arg("size"), pybind11::arg("timeout"));
}
