// harp_comm: NVLink peer-memory communication for 8xB200 (one process per GPU).
//
// Replaces the reference's communication layer: the HMPI c10d backend
// (hmpi/ProcessGroupHMPI.cpp:579-1234), the die-shared POSIX/SysV memory that
// ring attention and the gradient accumulator use (gemm/ring_attention/
// ring_attn.cpp:1344-1417, accumulate_sp/accumulate.cpp:63-387), and its
// unbounded spin flags (ring_attn.cpp:1871-1945).
//
//   * Symmetric heap: every rank cudaMalloc's the same segments in the same
//     order and maps every peer's segment through CUDA IPC, so a buffer has
//     the same offset on every rank and kernels address peers directly.
//   * Signals: a rank announces "my data for epoch e is ready" by storing e
//     with release semantics (system scope) into a flag slot in every peer's
//     flag segment; consumers wait with acquire loads, bounded by a timeout
//     that records an error word instead of hanging.  Only kernels wait for
//     flags written by OTHER GPUs; nothing on one GPU waits for another kernel
//     of the same GPU.
//   * Collectives are single kernels that pull peer data over NVLink with
//     16-byte loads and reduce/copy locally; the fused optimizer kernel
//     reduce-scatters gradients, runs AdamW and pushes the new bf16 shard into
//     every peer's parameter buffer with 16-byte stores.
#include "common.cuh"
#include "gemm_sm100.h"
#include "peer.cuh"

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <mutex>
#include <unordered_map>

namespace harp {
namespace comm {
namespace {

using bf16 = __nv_bfloat16;

struct Segment {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool owned = false;  // cudaMalloc'ed here (else an IPC mapping of a peer's segment)
  int device = 0;
};
std::mutex g_mu;
std::unordered_map<int64_t, Segment> g_segments;

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------

// flags[slot] on every peer (except `skip`) <- value, release at system scope.
__global__ void signal_kernel(PeerTable flags, int world, int slot, unsigned int value, int skip,
                              const int* step_delta, int per_step) {
  const int r = threadIdx.x;
  if (r >= world || r == skip) return;
  __threadfence_system();
  st_release_sys(reinterpret_cast<unsigned int*>(flags.base[r]) + slot, step_value(value, step_delta, per_step));
}

// Wait until local flags[first .. first+count) >= value.
__global__ void wait_kernel(const unsigned int* flags, int first, int count, unsigned int value,
                            unsigned long long timeout_ns, int* err, const int* step_delta, int per_step) {
  const int i = threadIdx.x;
  if (i >= count) return;
  wait_flag_geq(flags + first + i, step_value(value, step_delta, per_step), timeout_ns, err, 100 + i);
}

// Gather: for each source rank c (visited from rank+1 onwards), once
// flags[flag_first + c] >= value, copy `nseg` segments of `seg_bytes` from
// (src base of c) + src_off + s*src_stride to dst + c*dst_chunk_stride +
// s*dst_stride.  Source c == rank is read from local memory.  Bytes are
// multiples of 16 and every address 16-byte aligned.
__global__ void gather_kernel(PeerTable src, long long src_off, long long src_stride, char* __restrict__ dst,
                              long long dst_chunk_stride, long long dst_stride, long long seg_bytes, int nseg,
                              int world, int rank, const unsigned int* flags, int flag_first, unsigned int value,
                              unsigned long long timeout_ns, int* err) {
  const long long vec_per_seg = seg_bytes / 16;
  const long long vec_per_chunk = vec_per_seg * nseg;
  for (int step = 0; step < world; ++step) {
    const int c = (rank + step) % world;
    if (flags != nullptr && c != rank) {
      if (threadIdx.x == 0) wait_flag_geq(flags + flag_first + c, value, timeout_ns, err, 110 + c);
      __syncthreads();
      if (*(volatile int*)err != 0) return;
    }
    const char* sbase = reinterpret_cast<const char*>(src.base[c]) + src_off;
    char* dbase = dst + (long long)c * dst_chunk_stride;
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < vec_per_chunk;
         v += (long long)gridDim.x * blockDim.x) {
      const long long s = v / vec_per_seg, o = (v % vec_per_seg) * 16;
      const uint4 x = *reinterpret_cast<const uint4*>(sbase + s * src_stride + o);
      *reinterpret_cast<uint4*>(dbase + s * dst_stride + o) = x;
    }
  }
}

__device__ __forceinline__ void acc8(float (&a)[8], const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

// Reduce-scatter (pull): dst[n] = sum over ranks c of bf16 src_c[src_off + ...]
// where this rank's slice of every source consists of `nseg` segments of
// `seg_elems` at element stride `src_stride`; waits for each source's flag.
// Summation order is fixed (rank 0..world-1): every rank reduces identically.
__global__ void reduce_scatter_kernel(PeerTable src, long long src_off, long long src_stride, bf16* __restrict__ dst,
                                      long long dst_stride, long long seg_elems, int nseg, int world, int rank,
                                      const unsigned int* flags, int flag_first, unsigned int value,
                                      unsigned long long timeout_ns, int* err, const int* step_delta, int per_step) {
  if (flags != nullptr) {
    if (threadIdx.x < world && threadIdx.x != rank)
      wait_flag_geq(flags + flag_first + threadIdx.x, step_value(value, step_delta, per_step), timeout_ns, err,
                    120 + threadIdx.x);
    __syncthreads();
    if (*(volatile int*)err != 0) return;
  }
  const long long vec_per_seg = seg_elems / 8;
  const long long total = vec_per_seg * nseg;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const long long s = v / vec_per_seg, o = (v % vec_per_seg) * 8;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < world; ++c) {
      const bf16* sp = reinterpret_cast<const bf16*>(src.base[c]) + src_off + s * src_stride + o;
      acc8(a, *reinterpret_cast<const uint4*>(sp));
    }
    uint4 out;
    out.x = pack_bf16x2(a[0], a[1]);
    out.y = pack_bf16x2(a[2], a[3]);
    out.z = pack_bf16x2(a[4], a[5]);
    out.w = pack_bf16x2(a[6], a[7]);
    *reinterpret_cast<uint4*>(dst + s * dst_stride + o) = out;
  }
}

struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale;
};

// Fused optimizer step over NVLink for this rank's shard [lo, lo + n) of the
// flat buffers (n % 8 == 0):
//   g      = sum over ranks c of grad_c[lo + i]            (pull, fixed order)
//   master, m, v <- AdamW(master, m, v, g)                 (fp32, local shard)
//   param_c[lo + i] = bf16(master) for every rank c        (push)
// Waits first for every peer's "gradients ready" flag.
// local_out != nullptr (sharded parameters): the new bf16 slice is written
// there (local_out[i - lo]) instead of being pushed to every rank.
__global__ void rs_adamw_ag_kernel(PeerTable grads, PeerTable params, long long lo, long long n,
                                   float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                                   AdamHyper h, int world, int rank, const unsigned int* flags, int flag_first,
                                   unsigned int value, unsigned long long timeout_ns, int* err,
                                   bf16* __restrict__ local_out, const int* step_delta, int per_step,
                                   const float* __restrict__ hyper) {
  if (flags != nullptr) {
    if (threadIdx.x < world && threadIdx.x != rank)
      wait_flag_geq(flags + flag_first + threadIdx.x, step_value(value, step_delta, per_step), timeout_ns, err,
                    130 + threadIdx.x);
    __syncthreads();
    if (*(volatile int*)err != 0) return;
  }
  if (hyper != nullptr) {  // [lr, 1 - beta1^t, sqrt(1 - beta2^t)] of this step, on the device
    h.lr = hyper[0];
    h.bc1 = hyper[1];
    h.bc2_sqrt = hyper[2];
  }
  const long long nv = n / 8;
  for (long long vi = (long long)blockIdx.x * blockDim.x + threadIdx.x; vi < nv;
       vi += (long long)gridDim.x * blockDim.x) {
    const long long i = lo + vi * 8;
    float g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < world; ++c) acc8(g, *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(grads.base[c]) + i));
    float p[8];
    const long long li = vi * 8;
    float4 pm0 = *reinterpret_cast<const float4*>(master + li), pm1 = *reinterpret_cast<const float4*>(master + li + 4);
    float4 mm0 = *reinterpret_cast<const float4*>(m + li), mm1 = *reinterpret_cast<const float4*>(m + li + 4);
    float4 vv0 = *reinterpret_cast<const float4*>(v + li), vv1 = *reinterpret_cast<const float4*>(v + li + 4);
    float pa[8] = {pm0.x, pm0.y, pm0.z, pm0.w, pm1.x, pm1.y, pm1.z, pm1.w};
    float ma[8] = {mm0.x, mm0.y, mm0.z, mm0.w, mm1.x, mm1.y, mm1.z, mm1.w};
    float va[8] = {vv0.x, vv0.y, vv0.z, vv0.w, vv1.x, vv1.y, vv1.z, vv1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gg = g[j] * h.grad_scale;
      float pp = pa[j] * (1.f - h.lr * h.wd);
      const float mj = h.beta1 * ma[j] + (1.f - h.beta1) * gg;
      const float vj = h.beta2 * va[j] + (1.f - h.beta2) * gg * gg;
      pp -= (h.lr / h.bc1) * mj / (sqrtf(vj) / h.bc2_sqrt + h.eps);
      pa[j] = pp;
      ma[j] = mj;
      va[j] = vj;
      p[j] = pp;
    }
    *reinterpret_cast<float4*>(master + li) = make_float4(pa[0], pa[1], pa[2], pa[3]);
    *reinterpret_cast<float4*>(master + li + 4) = make_float4(pa[4], pa[5], pa[6], pa[7]);
    *reinterpret_cast<float4*>(m + li) = make_float4(ma[0], ma[1], ma[2], ma[3]);
    *reinterpret_cast<float4*>(m + li + 4) = make_float4(ma[4], ma[5], ma[6], ma[7]);
    *reinterpret_cast<float4*>(v + li) = make_float4(va[0], va[1], va[2], va[3]);
    *reinterpret_cast<float4*>(v + li + 4) = make_float4(va[4], va[5], va[6], va[7]);
    uint4 out;
    out.x = pack_bf16x2(p[0], p[1]);
    out.y = pack_bf16x2(p[2], p[3]);
    out.z = pack_bf16x2(p[4], p[5]);
    out.w = pack_bf16x2(p[6], p[7]);
    if (local_out != nullptr) {
      *reinterpret_cast<uint4*>(local_out + li) = out;
    } else {
      for (int c = 0; c < world; ++c) {
        const int dst = (rank + c) % world;  // stagger destinations across ranks
        *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(params.base[dst]) + i) = out;
      }
    }
  }
  __threadfence_system();
}

// All-gather push: n bf16 elements from local src into dst_c + off of every
// rank c (16-byte vectors, destinations staggered by rank), then a
// system-scope fence; the host follows with a release-store signal.
__global__ void push_slice_kernel(const bf16* __restrict__ src, PeerTable dst, long long off, long long n, int world,
                                  int rank) {
  const long long nv = n / 8;
  for (int c = 0; c < world; ++c) {
    const int d = (rank + 1 + c) % world;
    bf16* out = reinterpret_cast<bf16*>(dst.base[d]) + off;
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (long long)gridDim.x * blockDim.x)
      reinterpret_cast<uint4*>(out)[v] = reinterpret_cast<const uint4*>(src)[v];
  }
  __threadfence_system();
}


}  // namespace

// ---------------------------------------------------------------------------
// host API
// ---------------------------------------------------------------------------
std::tuple<int64_t, at::Tensor> ipc_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  std::lock_guard<std::mutex> lock(g_mu);
  g_segments[(int64_t)p] = Segment{p, (size_t)bytes, true, (int)device};
  return {(int64_t)p, t};
}

int64_t ipc_open(const at::Tensor& handle, int64_t device) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "harp_comm: bad IPC handle");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.cpu().contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  std::lock_guard<std::mutex> lock(g_mu);
  g_segments[(int64_t)p] = Segment{p, 0, false, (int)device};
  return (int64_t)p;
}

void ipc_release(int64_t ptr) {
  Segment s;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_segments.find(ptr);
    if (it == g_segments.end()) return;
    s = it->second;
    g_segments.erase(it);
  }
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)s.device);
  if (s.owned) cudaFree(s.ptr);
  else cudaIpcCloseMemHandle(s.ptr);
}

at::Tensor view(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, (c10::DeviceIndex)device));
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

const int* sd_ptr(const c10::optional<at::Tensor>& step_delta) {
  if (!step_delta.has_value()) return nullptr;
  TORCH_CHECK(step_delta->is_cuda() && step_delta->scalar_type() == at::kInt, "harp_comm: step_delta int32 CUDA");
  return step_delta->data_ptr<int>();
}

void signal(const std::vector<int64_t>& flag_bases, int64_t slot, int64_t value, int64_t skip,
            const c10::optional<at::Tensor>& step_delta, int64_t per_step) {
  const int world = flag_bases.size();
  signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(make_table(flag_bases, 0), world, (int)slot,
                                                                 (unsigned)value, (int)skip, sd_ptr(step_delta),
                                                                 (int)per_step);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void wait(const at::Tensor& flags, int64_t first, int64_t count, int64_t value, double timeout_s, at::Tensor& err,
          const c10::optional<at::Tensor>& step_delta, int64_t per_step) {
  TORCH_CHECK(count <= 1024, "harp_comm: wait on at most 1024 flags");
  if (count <= 0) return;
  wait_kernel<<<1, (unsigned)((count + 31) / 32 * 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const unsigned int*>(flags.data_ptr()), (int)first, (int)count, (unsigned)value,
      (unsigned long long)(timeout_s * 1e9), err.data_ptr<int>(), sd_ptr(step_delta), (int)per_step);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void gather(const std::vector<int64_t>& src_bases, int64_t src_off, int64_t src_stride, at::Tensor& dst,
            int64_t dst_off, int64_t dst_chunk_stride, int64_t dst_stride, int64_t seg_bytes, int64_t nseg,
            int64_t rank, const c10::optional<at::Tensor>& flags, int64_t flag_first, int64_t value, double timeout_s,
            at::Tensor& err) {
  TORCH_CHECK(seg_bytes % 16 == 0 && src_off % 16 == 0 && src_stride % 16 == 0 && dst_stride % 16 == 0 &&
                  dst_chunk_stride % 16 == 0 && dst_off % 16 == 0,
              "harp_comm gather: 16-byte granularity");
  const int world = src_bases.size();
  const long long vecs = seg_bytes / 16 * nseg;
  const int threads = 512;
  gather_kernel<<<grid_for(vecs, threads), threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(src_bases, 0), src_off, src_stride, reinterpret_cast<char*>(dst.data_ptr()) + dst_off,
      dst_chunk_stride, dst_stride, seg_bytes, (int)nseg, world, (int)rank,
      flags.has_value() ? reinterpret_cast<const unsigned int*>(flags->data_ptr()) : nullptr, (int)flag_first,
      (unsigned)value, (unsigned long long)(timeout_s * 1e9), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void reduce_scatter(const std::vector<int64_t>& src_bases, int64_t src_off, int64_t src_stride, at::Tensor& dst,
                    int64_t dst_stride, int64_t seg_elems, int64_t nseg, int64_t rank,
                    const c10::optional<at::Tensor>& flags, int64_t flag_first, int64_t value, double timeout_s,
                    at::Tensor& err, const c10::optional<at::Tensor>& step_delta, int64_t per_step) {
  TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && seg_elems % 8 == 0 && src_off % 8 == 0 && src_stride % 8 == 0 &&
                  dst_stride % 8 == 0,
              "harp_comm reduce_scatter: bf16, 8-element granularity");
  const int world = src_bases.size();
  const int threads = 512;
  reduce_scatter_kernel<<<grid_for(seg_elems / 8 * nseg, threads), threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(src_bases, 0), src_off, src_stride, reinterpret_cast<bf16*>(dst.data_ptr()), dst_stride, seg_elems,
      (int)nseg, world, (int)rank,
      flags.has_value() ? reinterpret_cast<const unsigned int*>(flags->data_ptr()) : nullptr, (int)flag_first,
      (unsigned)value, (unsigned long long)(timeout_s * 1e9), err.data_ptr<int>(), sd_ptr(step_delta),
      (int)per_step);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void rs_adamw_ag(const std::vector<int64_t>& grad_bases, const std::vector<int64_t>& param_bases, int64_t lo, int64_t n,
                 at::Tensor& master, at::Tensor& m, at::Tensor& v, double lr, double beta1, double beta2, double eps,
                 double wd, int64_t step, double grad_scale, int64_t rank, const c10::optional<at::Tensor>& flags,
                 int64_t flag_first, int64_t value, double timeout_s, at::Tensor& err, int64_t blocks,
                 const c10::optional<at::Tensor>& local_out, const c10::optional<at::Tensor>& step_delta,
                 int64_t per_step, const c10::optional<at::Tensor>& hyper) {
  if (hyper.has_value())
    TORCH_CHECK(hyper->is_cuda() && hyper->scalar_type() == at::kFloat && hyper->numel() >= 3,
                "harp_comm rs_adamw_ag: hyper fp32 [3] on the device");
  TORCH_CHECK(n % 8 == 0 && lo % 8 == 0, "harp_comm rs_adamw_ag: 8-element granularity");
  TORCH_CHECK(master.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "harp_comm rs_adamw_ag: contiguous state");
  TORCH_CHECK(master.numel() == n && m.numel() == n && v.numel() == n, "harp_comm rs_adamw_ag: state size");
  AdamHyper h;
  h.lr = lr; h.beta1 = beta1; h.beta2 = beta2; h.eps = eps; h.wd = wd;
  h.bc1 = 1.0 - std::pow(beta1, (double)step);
  h.bc2_sqrt = std::sqrt(1.0 - std::pow(beta2, (double)step));
  h.grad_scale = grad_scale;
  const int world = grad_bases.size();
  const int threads = 256;
  // blocks > 0 caps the grid (the kernel is grid-stride), so that a bucket's
  // kernel running beside the backward occupies only a few SMs
  int grid = grid_for(n / 8, threads);
  if (blocks > 0 && grid > blocks) grid = (int)blocks;
  if (n == 0) return;
  rs_adamw_ag_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(grad_bases, 0), make_table(param_bases, 0), lo, n, master.data_ptr<float>(), m.data_ptr<float>(),
      v.data_ptr<float>(), h, world, (int)rank,
      flags.has_value() ? reinterpret_cast<const unsigned int*>(flags->data_ptr()) : nullptr, (int)flag_first,
      (unsigned)value, (unsigned long long)(timeout_s * 1e9), err.data_ptr<int>(),
      local_out.has_value() ? reinterpret_cast<bf16*>(local_out->data_ptr()) : nullptr, sd_ptr(step_delta),
      (int)per_step, hyper.has_value() ? hyper->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void push_slice(const at::Tensor& src, const std::vector<int64_t>& dst_bases, int64_t off, int64_t rank,
                int64_t blocks) {
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.numel() % 8 == 0 && off % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0,
              "harp_comm push_slice: contiguous bf16, 16-byte granularity");
  const long long n = src.numel();
  if (n == 0) return;
  int grid = grid_for(n / 8, 256);
  if (blocks > 0 && grid > blocks) grid = (int)blocks;
  push_slice_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(src.data_ptr()), make_table(dst_bases, 0), off, n, (int)dst_bases.size(),
      (int)rank);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace comm
}  // namespace harp

TORCH_LIBRARY(harp_comm, m) {
  m.def("ipc_alloc(int bytes, int device) -> (int, Tensor)");
  m.def("ipc_open(Tensor handle, int device) -> int");
  m.def("ipc_release(int ptr) -> ()");
  m.def("view(int ptr, int numel, ScalarType dtype, int device) -> Tensor");
  m.def("signal(int[] flag_bases, int slot, int value, int skip, Tensor? step_delta=None, int per_step=0) -> ()");
  m.def("wait(Tensor flags, int first, int count, int value, float timeout_s, Tensor(a!) err, "
        "Tensor? step_delta=None, int per_step=0) -> ()");
  m.def("gather(int[] src_bases, int src_off, int src_stride, Tensor(a!) dst, int dst_off, int dst_chunk_stride, "
        "int dst_stride, int seg_bytes, int nseg, int rank, Tensor? flags, int flag_first, int value, float timeout_s, "
        "Tensor(b!) err) -> ()");
  m.def("reduce_scatter(int[] src_bases, int src_off, int src_stride, Tensor(a!) dst, int dst_stride, int seg_elems, "
        "int nseg, int rank, Tensor? flags, int flag_first, int value, float timeout_s, Tensor(b!) err, "
        "Tensor? step_delta=None, int per_step=0) -> ()");
  m.def("rs_adamw_ag(int[] grad_bases, int[] param_bases, int lo, int n, Tensor(a!) master, Tensor(b!) m, "
        "Tensor(c!) v, float lr, float beta1, float beta2, float eps, float wd, int step, float grad_scale, int rank, "
        "Tensor? flags, int flag_first, int value, float timeout_s, Tensor(d!) err, int blocks=0, "
        "Tensor(e!)? local_out=None, Tensor? step_delta=None, int per_step=0, Tensor? hyper=None) -> ()");
  m.def("push_slice(Tensor src, int[] dst_bases, int off, int rank, int blocks=0) -> ()");
}
TORCH_LIBRARY_IMPL(harp_comm, CompositeExplicitAutograd, m) {
  m.impl("ipc_alloc", &harp::comm::ipc_alloc);
  m.impl("ipc_open", &harp::comm::ipc_open);
  m.impl("ipc_release", &harp::comm::ipc_release);
  m.impl("view", &harp::comm::view);
  m.impl("signal", &harp::comm::signal);
}
TORCH_LIBRARY_IMPL(harp_comm, CUDA, m) {
  m.impl("wait", &harp::comm::wait);
  m.impl("gather", &harp::comm::gather);
  m.impl("reduce_scatter", &harp::comm::reduce_scatter);
  m.impl("rs_adamw_ag", &harp::comm::rs_adamw_ag);
  m.impl("push_slice", &harp::comm::push_slice);
}
